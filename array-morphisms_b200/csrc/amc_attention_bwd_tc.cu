// Tensor-core attention backward (sm_100a, tcgen05 kind::tf32), head dim 64.
//
// The reference has no attention gradient (grad.scm and ssa-vjp carry no
// rule for attention-morphism, blas-exec.scm:334-398); this is the standard
// softmax-attention VJP, with P rebuilt from the forward's row log-sum-exp:
//   P  = exp(scale * Q K^T - lse)           D  = rowsum(dO * O)
//   dP = dO V^T                             dS = P * (dP - D)
//   dV = P^T dO      dK = scale * dS^T Q    dQ = scale * dS K
// Two kernels, neither with atomics, so results are run-to-run identical:
//   k_attn_bwd_dkv_tc  one CTA per 128 keys (K, V resident); streams 64-query
//                      tiles: S^T = K Q^T, dP^T = V dO^T (tensor memory),
//                      the threads (one per key) form P^T and dS^T and write
//                      them back over S^T / dP^T, then dV += P^T dO and
//                      dK += dS^T Q take them as the A operand from TMEM;
//   k_attn_bwd_dq_tc   one CTA per 128 queries (Q, dO resident in tensor
//                      memory as the A operands); streams 64-key tiles:
//                      S, dP, dS as above, dQ += dS K.
// A pre-pass writes tf32-rounded copies of Q, K, V, dO and the per-row
// (lse * log2 e, D) pairs.  The S/dP products read K-major tiles of those
// copies (128-byte swizzle).  The products whose contraction runs over
// queries or keys (dV, dK: over queries; dQ: over keys) read the same rows
// as MN-major operands: a second tensor map with the 128-byte swizzle in
// 32-byte atoms, the only MN-major layout tf32 products accept.  No
// transposed copy is written.
// S/dP tensor-memory buffers (three in the dK/dV kernel, two in the dQ
// kernel, whose other columns hold Q and dO) let the products of the next
// tiles run while the threads work on the current one; two warpgroups share
// each tile, one taking its first 32 columns, the other the last 32.  One
// warp issues the S/dP products, another the accumulating ones.  Every wait
// is bounded; on expiry the kernel records AMC_ERR_TIMEOUT, drains and
// returns.
#include <cmath>
#include <mutex>
#include <unordered_map>

#include "amc_internal.h"
#include "amc_tc.cuh"

namespace amc {

using namespace tc;

namespace {

constexpr int kD = 64;        // head dim
constexpr int kTile = 128;    // keys (dK/dV) or queries (dQ) per CTA
constexpr int kStream = 64;   // streamed queries (dK/dV) or keys (dQ) per step
constexpr int kThreadsB = 384;   // warps 0-7 rows (two warpgroups), 8 and 9 producers, 10 and 11 MMA issuers
constexpr int kRowThreads = 256;

// dK/dV kernel shared memory (bytes from a 1024-aligned base)
constexpr int kKVK = 0;                          // K tile, 2 x 16 KB (dims 0-31, 32-63)
constexpr int kKVV = 32768;                      // V tile
constexpr int kKVF = 65536;                      // 3 stages x (Q_i 16 KB + dO_i 16 KB)
constexpr int kKVB = kKVF + 3 * 32768;           // 2 stages x (Q_i 16 KB + dO_i 16 KB), MN-major
constexpr int kKVL = kKVB + 2 * 32768;           // 3 stages x 64 (lse2, D) pairs
constexpr int kKVBar = kKVL + 3 * 512;
constexpr int kKVSmem = kKVBar + 256 + 1024;

// dQ kernel shared memory
constexpr int kQQ = 0;                           // Q tile, 2 x 16 KB
constexpr int kQdO = 32768;                      // dO tile
constexpr int kQF = 65536;                       // 3 stages x (K_j 16 KB + V_j 16 KB)
constexpr int kQB = kQF + 3 * 32768;             // 2 stages x K_j 16 KB, MN-major
constexpr int kQBar = kQB + 2 * 16384;
constexpr int kQSmem = kQBar + 256 + 1024;

static_assert(kKVSmem <= 232448, "dK/dV shared memory");
static_assert(kQSmem <= 232448, "dQ shared memory");

__device__ int g_attn_bwd_error;

}  // namespace

// ------------------------------------------------------------------ pre-pass
// One block per 32 rows of one (batch, head) block: rounded copies of Q, K,
// V, dO; LD[row] = (lse * log2 e, sum_d dO * O).
__global__ void __launch_bounds__(256) k_attn_bwd_prep(const float* __restrict__ Q, const float* __restrict__ K,
                                                       const float* __restrict__ V, const float* __restrict__ O,
                                                       const float* __restrict__ dO, const float* __restrict__ lse,
                                                       float* __restrict__ Qr, float* __restrict__ Kr,
                                                       float* __restrict__ Vr, float* __restrict__ dOr,
                                                       float2* __restrict__ LD, int n) {
  const int tid = threadIdx.x;
  const int bh = blockIdx.y, r0 = blockIdx.x * 32;
  const size_t base4 = ((size_t)bh * n + r0) * (kD / 4);
  const float4* src[3] = {reinterpret_cast<const float4*>(Q) + base4, reinterpret_cast<const float4*>(K) + base4,
                          reinterpret_cast<const float4*>(dO) + base4};
  float4* dst[3] = {reinterpret_cast<float4*>(Qr) + base4, reinterpret_cast<float4*>(Kr) + base4,
                    reinterpret_cast<float4*>(dOr) + base4};
#pragma unroll
  for (int it = 0; it < 2; ++it) {
    const int i = tid + it * 256;        // float4 index in the 32 x 64 tile
    const int row = i >> 4, c = (i & 15) * 4;
#pragma unroll
    for (int a = 0; a < 3; ++a) {
      const float4 v = src[a][i];
      dst[a][i] = make_float4(round_tf32(v.x), round_tf32(v.y), round_tf32(v.z), round_tf32(v.w));
    }
    const float4 v = reinterpret_cast<const float4*>(V)[base4 + i];
    reinterpret_cast<float4*>(Vr)[base4 + i] =
        make_float4(round_tf32(v.x), round_tf32(v.y), round_tf32(v.z), round_tf32(v.w));
    // D: 16 consecutive threads cover one row
    const float4 g = src[2][i];
    const float4 o = reinterpret_cast<const float4*>(O)[base4 + i];
    float d = g.x * o.x + g.y * o.y + g.z * o.z + g.w * o.w;
#pragma unroll
    for (int off = 8; off > 0; off >>= 1) d += __shfl_xor_sync(0xffffffffu, d, off);
    if ((i & 15) == 0) {
      const size_t r = (size_t)bh * n + r0 + row;
      LD[r] = make_float2(lse[r] * 1.4426950408889634f, d);
    }
  }
}

// ------------------------------------------------------------------ dK, dV
__global__ void __launch_bounds__(kThreadsB, 1) k_attn_bwd_dkv_tc(
    const __grid_constant__ CUtensorMap mK, const __grid_constant__ CUtensorMap mV,
    const __grid_constant__ CUtensorMap mQ, const __grid_constant__ CUtensorMap mdO,
    const __grid_constant__ CUtensorMap mQmn, const __grid_constant__ CUtensorMap mdOmn,
    const float2* __restrict__ LD, float* __restrict__ dK, float* __restrict__ dV, int n, float scale_log2,
    float scale) {
  extern __shared__ unsigned char bkv_sm_raw[];
  unsigned char* sm = (unsigned char*)(((uintptr_t)bkv_sm_raw + 1023) & ~(uintptr_t)1023);
  uint64_t* kv_full = (uint64_t*)(sm + kKVBar);
  uint64_t* f_full = kv_full + 1;    // [3] Q_i, dO_i, LD_i landed
  uint64_t* f_empty = kv_full + 4;   // [3] S/dP products done and LD read
  uint64_t* b_full = kv_full + 7;    // [2] MN-major Q_i, dO_i landed
  uint64_t* b_empty = kv_full + 9;   // [2]
  uint64_t* s_full = kv_full + 11;   // [3] S^T, dP^T in tensor memory
  uint64_t* p_full = kv_full + 14;   // [3] P^T, dS^T written back
  uint64_t* t_free = kv_full + 17;   // [3] dV/dK products read the buffer
  uint64_t* acc_full = kv_full + 20;
  uint32_t* tslot = (uint32_t*)(sm + kKVBar + 192);
  volatile int* abort_flag = (volatile int*)(sm + kKVBar + 196);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int bh = blockIdx.y;
  const int key0 = bh * n + blockIdx.x * kTile;
  const int nt = n / kStream;
  if (tid == 0) {
    mbar_init(kv_full, 1);
    for (int i = 0; i < 3; ++i) {
      mbar_init(&f_full[i], 1);
      mbar_init(&f_empty[i], 1 + kRowThreads);
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], kRowThreads);
      mbar_init(&t_free[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&b_full[i], 1);
      mbar_init(&b_empty[i], 1);
    }
    mbar_init(acc_full, 1);
    *abort_flag = 0;
    mbar_fence_init();
  }
  __syncthreads();
  if (warp == 0) tmem_alloc(tslot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;
  const uint32_t t_dv = tmem + 384, t_dk = tmem + 448;

  if (warp == 8) {
    if (lane == 0) {
      mbar_expect_tx(kv_full, 4 * 16384);
      for (int r = 0; r < 2; ++r) {
        tma_load_2d(sm + kKVK + r * 16384, &mK, 32 * r, key0, kv_full);
        tma_load_2d(sm + kKVV + r * 16384, &mV, 32 * r, key0, kv_full);
      }
      for (int i = 0; i < nt; ++i) {
        const int s = i % 3;
        if (i >= 3 && !mbar_wait(&f_empty[s], (uint32_t)((i - 3) / 3) & 1u)) { *abort_flag = 1; break; }
        if (*abort_flag) break;
        const int q0 = bh * n + i * kStream;
        unsigned char* st = sm + kKVF + s * 32768;
        mbar_expect_tx(&f_full[s], 32768 + 512);
        for (int r = 0; r < 2; ++r) {
          tma_load_2d(st + r * 8192, &mQ, 32 * r, q0, &f_full[s]);
          tma_load_2d(st + 16384 + r * 8192, &mdO, 32 * r, q0, &f_full[s]);
        }
        bulk_load_1d(sm + kKVL + s * 512, LD + q0, 512, &f_full[s]);
      }
    }
  } else if (warp == 9) {
    if (lane == 0) {
      for (int i = 0; i < nt; ++i) {
        const int b = i & 1;
        if (i >= 2 && !mbar_wait(&b_empty[b], (uint32_t)((i - 2) >> 1) & 1u)) { *abort_flag = 1; break; }
        if (*abort_flag) break;
        unsigned char* st = sm + kKVB + b * 32768;
        mbar_expect_tx(&b_full[b], 32768);
        for (int r = 0; r < 2; ++r) {
          tma_load_2d(st + r * 8192, &mQmn, 32 * r, bh * n + i * kStream, &b_full[b]);
          tma_load_2d(st + 16384 + r * 8192, &mdOmn, 32 * r, bh * n + i * kStream, &b_full[b]);
        }
      }
    }
  } else if (warp >= 10) {
    // warp 10 issues the S/dP products, warp 11 the accumulating ones
    if (lane == 0) {
      const uint32_t id = idesc_tf32(kTile, 64, false, false);
      const uint32_t id_mn = idesc_tf32(kTile, 64, false, true);   // B MN-major
      const uint64_t dk0 = sdesc(smem_addr(sm + kKVK), 16, 1024), dv0 = sdesc(smem_addr(sm + kKVV), 16, 1024);
      // B-stage: region r (8 KB) holds dims 32r..32r+31 of 64 query rows
      const uint64_t df0 = sdesc(smem_addr(sm + kKVF), 16, 1024), db0 = sdesc_mn(smem_addr(sm + kKVB), 8192);
      // S^T = K Q_i^T and dP^T = V dO_i^T into buffer i % 3
      auto sdp = [&](int i) -> bool {
        const int s = i % 3;
        if (!mbar_wait(&f_full[s], (uint32_t)(i / 3) & 1u)) return false;
        if (i >= 3 && !mbar_wait(&t_free[s], (uint32_t)((i - 3) / 3) & 1u)) return false;
        tc_fence_after();
        const uint32_t ts = tmem + s * 128;
        const uint64_t st = desc_add(df0, s * 32768);
#pragma unroll
        for (int k = 0; k < kD / 8; ++k) {
          mma_tf32(ts, desc_add(dk0, kstep_off(k, 16384)), desc_add(st, kstep_off(k, 8192)), id, k > 0);
          mma_tf32(ts + 64, desc_add(dv0, kstep_off(k, 16384)), desc_add(st, 16384 + kstep_off(k, 8192)), id, k > 0);
        }
        mma_commit(&s_full[s]);
        mma_commit(&f_empty[s]);
        return true;
      };
      // dV += P^T dO_i, dK += dS^T Q_i (A operands from tensor memory; B
      // MN-major, K step k = query rows 8k..8k+7)
      auto dvdk = [&](int i) -> bool {
        const int s = i % 3, b = i & 1;
        if (!mbar_wait(&p_full[s], (uint32_t)(i / 3) & 1u)) return false;
        if (!mbar_wait(&b_full[b], (uint32_t)(i >> 1) & 1u)) return false;
        tc_fence_after();
        const uint32_t ts = tmem + s * 128;
        const uint64_t st = desc_add(db0, b * 32768);
        const bool acc0 = i > 0;
#pragma unroll
        for (int k = 0; k < kStream / 8; ++k) {
          mma_tf32_ts(t_dv, ts + k * 8, desc_add(st, 16384 + k * 1024), id_mn, acc0 || k > 0);
          mma_tf32_ts(t_dk, ts + 64 + k * 8, desc_add(st, k * 1024), id_mn, acc0 || k > 0);
        }
        mma_commit(&b_empty[b]);
        mma_commit(&t_free[s]);
        return true;
      };
      bool ok = true;
      if (warp == 10) {
        ok = mbar_wait(kv_full, 0);
        for (int i = 0; i < nt && ok && !*abort_flag; ++i) ok = sdp(i);
      } else {
        for (int i = 0; i < nt && ok && !*abort_flag; ++i) ok = dvdk(i);
        if (ok) mma_commit(acc_full);
      }
      if (!ok) *abort_flag = 1;
    }
  } else if (warp < 8) {
    // one thread per key row of the tile; warpgroup g takes columns 32g..32g+31
    const int g = warp >> 2, t = tid & 127;
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
    bool ok = true;
    for (int i = 0; i < nt; ++i) {
      const int s = i % 3;
      const uint32_t ph = (uint32_t)(i / 3) & 1u;
      // (lse2, D) of this warpgroup's 32 query columns, two per 16-byte
      // broadcast load, fetched as soon as the stage has landed and before the
      // wait for S^T/dP^T, so their latency (the loads share the shared-memory
      // port with the tensor-core operand reads) is hidden behind that wait
      const bool landed = mbar_wait(&f_full[s], ph);
      const float4* ld = reinterpret_cast<const float4*>(sm + kKVL + s * 512) + 16 * g;
      float4 ev[16];
#pragma unroll
      for (int q = 0; q < 16; ++q) ev[q] = ld[q];
      mbar_arrive(&f_empty[s]);
      ok = named_bar_and(1, kRowThreads, landed && mbar_wait(&s_full[s], ph) && !*abort_flag);
      if (!ok) break;
      tc_fence_after();
      const uint32_t ts = tmem + s * 128 + lane_base + 32 * g;
      uint32_t sv[32], pv[32];
      tmem_ld32_nowait(ts, sv);
      tmem_ld32_nowait(ts + 64, pv);
      tmem_ld_wait();
      float po[32], dso[32];
#pragma unroll
      for (int j = 0; j < 32; j += 2) {
        const float4 e = ev[j >> 1];
        const float p0 = ex2_approx(fmaf(__uint_as_float(sv[j]), scale_log2, -e.x));
        const float p1 = ex2_approx(fmaf(__uint_as_float(sv[j + 1]), scale_log2, -e.z));
        po[j] = round_tf32_int(p0);
        po[j + 1] = round_tf32_int(p1);
        dso[j] = round_tf32_int(p0 * (__uint_as_float(pv[j]) - e.y));
        dso[j + 1] = round_tf32_int(p1 * (__uint_as_float(pv[j + 1]) - e.w));
      }
      tmem_st32(ts, po);
      tmem_st32(ts + 64, dso);
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(&p_full[s]);
    }
    if (ok) ok = named_bar_and(1, kRowThreads, mbar_wait(acc_full, 0) && !*abort_flag);
    if (ok) {
      // warpgroup 0 writes the dV row, warpgroup 1 the dK row
      tc_fence_after();
      const size_t row = (size_t)key0 + t;
      const float f = g ? scale : 1.f;
      float* dst = (g ? dK : dV) + row * kD;
      const uint32_t src = (g ? t_dk : t_dv) + lane_base;
#pragma unroll
      for (int c = 0; c < kD; c += 32) {
        float v[32];
        tmem_ld32(src + c, v);
        float4* o4 = reinterpret_cast<float4*>(dst + c);
#pragma unroll
        for (int j = 0; j < 8; ++j) o4[j] = make_float4(v[4 * j] * f, v[4 * j + 1] * f, v[4 * j + 2] * f, v[4 * j + 3] * f);
      }
    } else if (tid == 0) {
      *abort_flag = 1;
      atomicExch(&g_attn_bwd_error, AMC_ERR_TIMEOUT);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (*abort_flag) {
    if (tid == 0) atomicExch(&g_attn_bwd_error, AMC_ERR_TIMEOUT);
    // bounded drain of copies and products still in flight
    mbar_wait(kv_full, 0, 1 << 14);
    for (int i = 0; i < 3; ++i) {
      mbar_wait(&f_full[i], 0, 1 << 14);
      mbar_wait(&s_full[i], 0, 1 << 14);
      mbar_wait(&t_free[i], 0, 1 << 14);
    }
    for (int i = 0; i < 2; ++i) mbar_wait(&b_full[i], 0, 1 << 14);
  }
  if (warp == 0) tmem_dealloc(tmem, 512);
}

// ------------------------------------------------------------------ dQ
__global__ void __launch_bounds__(kThreadsB, 1) k_attn_bwd_dq_tc(
    const __grid_constant__ CUtensorMap mQ, const __grid_constant__ CUtensorMap mdO,
    const __grid_constant__ CUtensorMap mK, const __grid_constant__ CUtensorMap mV,
    const __grid_constant__ CUtensorMap mKmn, const float2* __restrict__ LD, float* __restrict__ dQ, int n,
    float scale_log2, float scale) {
  extern __shared__ unsigned char bq_sm_raw[];
  unsigned char* sm = (unsigned char*)(((uintptr_t)bq_sm_raw + 1023) & ~(uintptr_t)1023);
  uint64_t* qd_full = (uint64_t*)(sm + kQBar);
  uint64_t* f_full = qd_full + 1;    // [3] K_j, V_j landed
  uint64_t* f_empty = qd_full + 4;   // [3]
  uint64_t* b_full = qd_full + 7;    // [2] MN-major K_j landed
  uint64_t* b_empty = qd_full + 9;   // [2]
  uint64_t* s_full = qd_full + 11;   // [2] per tensor-memory buffer
  uint64_t* p_full = qd_full + 14;   // [2] dS written back
  uint64_t* t_free = qd_full + 17;   // [2]
  uint64_t* acc_full = qd_full + 20;
  uint64_t* qd_ready = qd_full + 21; // Q and dO rows in tensor memory
  uint32_t* tslot = (uint32_t*)(sm + kQBar + 192);
  volatile int* abort_flag = (volatile int*)(sm + kQBar + 196);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int bh = blockIdx.y;
  const int q0 = bh * n + blockIdx.x * kTile;
  const int nt = n / kStream;
  if (tid == 0) {
    mbar_init(qd_full, 1);
    for (int i = 0; i < 3; ++i) {
      mbar_init(&f_full[i], 1);
      mbar_init(&f_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], kRowThreads);
      mbar_init(&t_free[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&b_full[i], 1);
      mbar_init(&b_empty[i], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(qd_ready, kRowThreads);
    *abort_flag = 0;
    mbar_fence_init();
  }
  __syncthreads();
  if (warp == 0) tmem_alloc(tslot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;
  // S/dP buffers at 0 and 128, dQ at 256, Q at 320, dO at 384 (the A
  // operands of the S and dP products, so those read only K_j and V_j from
  // shared memory)
  const uint32_t t_dq = tmem + 256, t_q = tmem + 320, t_do = tmem + 384;

  if (warp == 8) {
    if (lane == 0) {
      mbar_expect_tx(qd_full, 4 * 16384);
      for (int r = 0; r < 2; ++r) {
        tma_load_2d(sm + kQQ + r * 16384, &mQ, 32 * r, q0, qd_full);
        tma_load_2d(sm + kQdO + r * 16384, &mdO, 32 * r, q0, qd_full);
      }
      for (int j = 0; j < nt; ++j) {
        const int s = j % 3;
        if (j >= 3 && !mbar_wait(&f_empty[s], (uint32_t)((j - 3) / 3) & 1u)) { *abort_flag = 1; break; }
        if (*abort_flag) break;
        const int k0 = bh * n + j * kStream;
        unsigned char* st = sm + kQF + s * 32768;
        mbar_expect_tx(&f_full[s], 32768);
        for (int r = 0; r < 2; ++r) {
          tma_load_2d(st + r * 8192, &mK, 32 * r, k0, &f_full[s]);
          tma_load_2d(st + 16384 + r * 8192, &mV, 32 * r, k0, &f_full[s]);
        }
      }
    }
  } else if (warp == 9) {
    if (lane == 0) {
      for (int j = 0; j < nt; ++j) {
        const int b = j & 1;
        if (j >= 2 && !mbar_wait(&b_empty[b], (uint32_t)((j - 2) >> 1) & 1u)) { *abort_flag = 1; break; }
        if (*abort_flag) break;
        unsigned char* st = sm + kQB + b * 16384;
        mbar_expect_tx(&b_full[b], 16384);
        for (int r = 0; r < 2; ++r) tma_load_2d(st + r * 8192, &mKmn, 32 * r, bh * n + j * kStream, &b_full[b]);
      }
    }
  } else if (warp >= 10) {
    // warp 10 issues the S/dP products, warp 11 the accumulating ones
    if (lane == 0) {
      const uint32_t id = idesc_tf32(kTile, 64, false, false);
      const uint32_t id_mn = idesc_tf32(kTile, 64, false, true);   // B MN-major
      const uint64_t df0 = sdesc(smem_addr(sm + kQF), 16, 1024), db0 = sdesc_mn(smem_addr(sm + kQB), 8192);
      // S = Q K_j^T, dP = dO V_j^T into buffer j % 2; K_j, V_j from stage j % 3
      auto sdp = [&](int j) -> bool {
        const int f = j % 3, s = j & 1;
        if (!mbar_wait(&f_full[f], (uint32_t)(j / 3) & 1u)) return false;
        if (j >= 2 && !mbar_wait(&t_free[s], (uint32_t)((j - 2) >> 1) & 1u)) return false;
        tc_fence_after();
        const uint32_t ts = tmem + s * 128;
        const uint64_t st = desc_add(df0, f * 32768);
#pragma unroll
        for (int k = 0; k < kD / 8; ++k) {
          mma_tf32_ts(ts, t_q + k * 8, desc_add(st, kstep_off(k, 8192)), id, k > 0);
          mma_tf32_ts(ts + 64, t_do + k * 8, desc_add(st, 16384 + kstep_off(k, 8192)), id, k > 0);
        }
        mma_commit(&s_full[s]);
        mma_commit(&f_empty[f]);
        return true;
      };
      auto dq = [&](int j) -> bool {
        const int s = j & 1, b = j & 1;
        if (!mbar_wait(&p_full[s], (uint32_t)(j >> 1) & 1u)) return false;
        if (!mbar_wait(&b_full[b], (uint32_t)(j >> 1) & 1u)) return false;
        tc_fence_after();
        const uint32_t ts = tmem + s * 128;
        const uint64_t st = desc_add(db0, b * 16384);
        const bool acc0 = j > 0;
#pragma unroll
        for (int k = 0; k < kStream / 8; ++k) mma_tf32_ts(t_dq, ts + 64 + k * 8, desc_add(st, k * 1024), id_mn, acc0 || k > 0);
        mma_commit(&b_empty[b]);
        mma_commit(&t_free[s]);
        return true;
      };
      bool ok = true;
      if (warp == 10) {
        ok = mbar_wait(qd_ready, 0);
        for (int j = 0; j < nt && ok && !*abort_flag; ++j) ok = sdp(j);
      } else {
        for (int j = 0; j < nt && ok && !*abort_flag; ++j) ok = dq(j);
        if (ok) mma_commit(acc_full);
      }
      if (!ok) *abort_flag = 1;
    }
  } else if (warp < 8) {
    // one thread per query row of the tile; warpgroup g takes columns 32g..32g+31
    const int g = warp >> 2, t = tid & 127;
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
    const float2 e = LD[q0 + t];
    bool ok = mbar_wait(qd_full, 0);
    if (!ok) *abort_flag = 1;
    {
      // warpgroup 0 moves its Q row, warpgroup 1 its dO row (already rounded)
      // into tensor memory lane t; the staged rows are 128-byte swizzled
      const unsigned char* row = sm + (g ? kQdO : kQQ) + t * 128;
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        float v[32];
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const float4 x = *reinterpret_cast<const float4*>(row + r * 16384 + ((c ^ (t & 7)) << 4));
          v[4 * c] = x.x;
          v[4 * c + 1] = x.y;
          v[4 * c + 2] = x.z;
          v[4 * c + 3] = x.w;
        }
        tmem_st32((g ? t_do : t_q) + lane_base + 32 * r, v);
      }
      tmem_st_wait();
      tc_fence_before();
    }
    mbar_arrive(qd_ready);
    for (int j = 0; j < nt; ++j) {
      const int s = j & 1;
      ok = named_bar_and(1, kRowThreads, ok && mbar_wait(&s_full[s], (uint32_t)(j >> 1) & 1u) && !*abort_flag);
      if (!ok) break;
      tc_fence_after();
      const uint32_t ts = tmem + s * 128 + lane_base + 32 * g;
      uint32_t sv[32], pv[32];
      tmem_ld32_nowait(ts, sv);
      tmem_ld32_nowait(ts + 64, pv);
      tmem_ld_wait();
      float dso[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const float p = ex2_approx(fmaf(__uint_as_float(sv[i]), scale_log2, -e.x));
        dso[i] = round_tf32_int(p * (__uint_as_float(pv[i]) - e.y));
      }
      tmem_st32(ts + 64, dso);
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(&p_full[s]);
    }
    if (ok) ok = named_bar_and(1, kRowThreads, mbar_wait(acc_full, 0) && !*abort_flag);
    if (ok) {
      // warpgroup g writes dQ columns 32g..32g+31
      tc_fence_after();
      const size_t row = (size_t)q0 + t;
      float v[32];
      tmem_ld32(t_dq + lane_base + 32 * g, v);
      float4* dqr = reinterpret_cast<float4*>(dQ + row * kD + 32 * g);
#pragma unroll
      for (int i = 0; i < 8; ++i)
        dqr[i] = make_float4(v[4 * i] * scale, v[4 * i + 1] * scale, v[4 * i + 2] * scale, v[4 * i + 3] * scale);
    } else if (tid == 0) {
      *abort_flag = 1;
      atomicExch(&g_attn_bwd_error, AMC_ERR_TIMEOUT);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (*abort_flag) {
    if (tid == 0) atomicExch(&g_attn_bwd_error, AMC_ERR_TIMEOUT);
    mbar_wait(qd_full, 0, 1 << 14);
    for (int i = 0; i < 3; ++i) {
      mbar_wait(&f_full[i], 0, 1 << 14);
      mbar_wait(&s_full[i], 0, 1 << 14);
      mbar_wait(&t_free[i], 0, 1 << 14);
    }
    for (int i = 0; i < 2; ++i) mbar_wait(&b_full[i], 0, 1 << 14);
  }
  if (warp == 0) tmem_dealloc(tmem, 512);
}

// ------------------------------------------------------------------ host
// Per-device scratch for the pre-pass outputs, grown on demand and kept.
static int bwd_scratch(size_t bytes, void** out) {
  static std::mutex mu;
  static std::unordered_map<int, std::pair<void*, size_t>> bufs;
  int dev = 0;
  AMC_CUDA(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> l(mu);
  auto& e = bufs[dev];
  if (e.second < bytes) {
    if (e.first) {
      AMC_CUDA(cudaDeviceSynchronize());
      cudaFree(e.first);
      e = {nullptr, 0};
    }
    AMC_CUDA(cudaMalloc(&e.first, bytes));
    e.second = bytes;
  }
  *out = e.first;
  return AMC_OK;
}

int attention_bwd_tc(const float* Q, const float* K, const float* V, const float* O, const float* dO,
                     const float* lse, float* dQ, float* dK, float* dV, long long blocks, int n, int dk, int dv,
                     float scale, cudaStream_t s, bool* handled) {
  *handled = false;
  if (dk != kD || dv != kD || n < kTile || (n % kTile) != 0 || blocks <= 0 || blocks > 65535) return AMC_OK;
  if (((uintptr_t)Q | (uintptr_t)K | (uintptr_t)V | (uintptr_t)O | (uintptr_t)dO | (uintptr_t)dQ | (uintptr_t)dK |
       (uintptr_t)dV) & 15)
    return AMC_OK;
  const uint64_t rows = (uint64_t)blocks * n;
  if (rows > 0x7fffffffull) return AMC_OK;
  *handled = true;
  const size_t telems = (size_t)rows * kD;
  float* scr = nullptr;
  int rc = bwd_scratch((4 * telems + 2 * rows) * sizeof(float), (void**)&scr);
  if (rc) return rc;
  float *Qr = scr, *Kr = Qr + telems, *Vr = Kr + telems, *dOr = Vr + telems;
  float2* LD = reinterpret_cast<float2*>(dOr + telems);
  k_attn_bwd_prep<<<dim3(n / 32, (unsigned)blocks), 256, 0, s>>>(Q, K, V, O, dO, lse, Qr, Kr, Vr, dOr, LD, n);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "k_attn_bwd_prep");
  CUtensorMap mK128, mV128, mQ64, mdO64, mQmn, mdOmn, mQ128, mdO128, mK64, mV64, mKmn;
  rc = make_tmap_2d_f32(&mK128, Kr, rows, kD, kD, 128);
  if (!rc) rc = make_tmap_2d_f32(&mV128, Vr, rows, kD, kD, 128);
  if (!rc) rc = make_tmap_2d_f32(&mQ64, Qr, rows, kD, kD, 64);
  if (!rc) rc = make_tmap_2d_f32(&mdO64, dOr, rows, kD, kD, 64);
  if (!rc) rc = make_tmap_2d_f32_swz(&mQmn, Qr, rows, kD, kD, 32, 64, TmapSwizzle::k128Atom32);
  if (!rc) rc = make_tmap_2d_f32_swz(&mdOmn, dOr, rows, kD, kD, 32, 64, TmapSwizzle::k128Atom32);
  if (!rc) rc = make_tmap_2d_f32(&mQ128, Qr, rows, kD, kD, 128);
  if (!rc) rc = make_tmap_2d_f32(&mdO128, dOr, rows, kD, kD, 128);
  if (!rc) rc = make_tmap_2d_f32(&mK64, Kr, rows, kD, kD, 64);
  if (!rc) rc = make_tmap_2d_f32(&mV64, Vr, rows, kD, kD, 64);
  if (!rc) rc = make_tmap_2d_f32_swz(&mKmn, Kr, rows, kD, kD, 32, 64, TmapSwizzle::k128Atom32);
  if (rc) return rc;
  static std::atomic<uint64_t> attr_dkv{0}, attr_dq{0};
  rc = smem_attr_once(k_attn_bwd_dkv_tc, kKVSmem, attr_dkv);
  if (!rc) rc = smem_attr_once(k_attn_bwd_dq_tc, kQSmem, attr_dq);
  if (rc) return rc;
  const float scale_log2 = scale * 1.4426950408889634f;
  const dim3 grid(n / kTile, (unsigned)blocks);
  k_attn_bwd_dkv_tc<<<grid, kThreadsB, kKVSmem, s>>>(mK128, mV128, mQ64, mdO64, mQmn, mdOmn, LD, dK, dV, n, scale_log2,
                                                     scale);
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "k_attn_bwd_dkv_tc");
  k_attn_bwd_dq_tc<<<grid, kThreadsB, kQSmem, s>>>(mQ128, mdO128, mK64, mV64, mKmn, LD, dQ, n, scale_log2, scale);
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "k_attn_bwd_dq_tc");
  return AMC_OK;
}

int attention_bwd_check_error() {
  int e = 0;
  AMC_CUDA(cudaMemcpyFromSymbol(&e, g_attn_bwd_error, sizeof(int)));
  if (e) {
    int z = 0;
    AMC_CUDA(cudaMemcpyToSymbol(g_attn_bwd_error, &z, sizeof(int)));
    return fail(e, "attention backward: a bounded wait on the tensor-core pipeline gave up");
  }
  return AMC_OK;
}

}  // namespace amc
