// Tensor-core attention forward (sm_100a, tcgen05 kind::tf32).
//
// Two kernels: k_attn_fwd_tc3 (below: 256 query rows per CTA, n a multiple of
// 256) and k_attn_fwd_tc for n a multiple of 128 only.  The latter:
// one CTA computes 128 query rows of one (batch, head) block, one thread per
// row.  For each 128-key tile:
//   S  = Q K^T      tcgen05.mma M=128 N=128 K=64, operands K-major in shared
//                   memory (TMA, 128-byte swizzle), accumulator in TMEM
//   P  = exp(scale*S - m) with the running row max m and sum l (online
//        softmax of the reference's 3-pass %attn-2d!, realization.scm:279-326)
//   O_t = P V       tcgen05.mma M=128 N=64 K=128; P is written by the threads
//                   into shared memory in the K-major swizzled layout; V is
//                   an MN-major operand (its rows are the contraction axis):
//                   the TMA writes it with the 128-byte swizzle in 32-byte
//                   atoms, the only MN-major layout tf32 products accept
//   O  = O * exp(m_old - m) + O_t   in registers
// K and V are read from tf32-rounded copies that one pre-pass writes.
// K and V tiles are double-buffered: the TMA for tile j+2 is issued as soon
// as the P V product of tile j has consumed its buffer.  Every mbarrier wait is
// bounded; on expiry the CTA records AMC_ERR_TIMEOUT and leaves after its MMAs
// and copies have drained.
#include <cmath>

#include "amc_internal.h"
#include "amc_tc.cuh"

namespace amc {

using namespace tc;

namespace {

constexpr int kBM = 128;   // query rows per CTA
constexpr int kBN = 128;   // keys per tile
constexpr int kD = 64;     // head dim

// shared memory map (bytes, from a 1024-aligned base)
constexpr int kQOff = 0;                         // 2 x 16 KB   (dims 0-31, 32-63)
constexpr int kKOff = kQOff + 2 * 16384;         // 2 bufs x 2 x 16 KB
constexpr int kVOff = kKOff + 2 * 2 * 16384;     // 2 bufs x 2 x 16 KB (dims 0-31, 32-63), 128 key rows each (MN-major)
constexpr int kPOff = kVOff + 2 * 4 * 8192;      // 4 x 16 KB   (keys 0-31 .. 96-127)
constexpr int kBarOff = kPOff + 4 * 16384;
constexpr int kSmemBytes = kBarOff + 128 + 1024; // barriers, tmem slot, alignment slack

__device__ int g_attn_error;

__device__ __forceinline__ void fail_timeout() { atomicExch(&g_attn_error, AMC_ERR_TIMEOUT); }

}  // namespace

__global__ void __launch_bounds__(128, 1) k_attn_fwd_tc(const __grid_constant__ CUtensorMap mQ,
                                                       const __grid_constant__ CUtensorMap mK,
                                                       const __grid_constant__ CUtensorMap mV, float* __restrict__ O,
                                                       float* __restrict__ lse, int n, float scale_log2) {
  extern __shared__ unsigned char attn_sm_raw[];
  unsigned char* sm = (unsigned char*)(((uintptr_t)attn_sm_raw + 1023) & ~(uintptr_t)1023);
  uint64_t* bar_q = (uint64_t*)(sm + kBarOff);
  uint64_t* bar_kv = bar_q + 1;   // [2]
  uint64_t* bar_s = bar_q + 3;
  uint64_t* bar_o = bar_q + 4;
  uint32_t* tslot = (uint32_t*)(sm + kBarOff + 64);
  const int tid = threadIdx.x, warp = tid >> 5;
  const int qtile = blockIdx.x, bh = blockIdx.y;
  const int row0 = bh * n + qtile * kBM;   // row in the (B*H*n, 64) view of Q / O
  const int ntiles = n / kBN;
  if (tid == 0) {
    mbar_init(bar_q, 1);
    mbar_init(&bar_kv[0], 1);
    mbar_init(&bar_kv[1], 1);
    mbar_init(bar_s, 1);
    mbar_init(bar_o, 1);
    mbar_fence_init();
  }
  __syncthreads();
  if (warp == 0) tmem_alloc(tslot, 256);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;
  const uint32_t t_s = tmem, t_o = tmem + 128;
  const uint32_t lane_base = (uint32_t)(warp * 32) << 16;

  auto load_kv = [&](int j, int b) {
    mbar_expect_tx(&bar_kv[b], 2 * 16384 + 4 * 8192);
    for (int r = 0; r < 2; ++r) tma_load_2d(sm + kKOff + b * 32768 + r * 16384, &mK, 32 * r, bh * n + j * kBN, &bar_kv[b]);
    for (int r = 0; r < 2; ++r) tma_load_2d(sm + kVOff + b * 32768 + r * 16384, &mV, 32 * r, bh * n + j * kBN, &bar_kv[b]);
  };
  if (tid == 0) {
    mbar_expect_tx(bar_q, 2 * 16384);
    for (int r = 0; r < 2; ++r) tma_load_2d(sm + kQOff + r * 16384, &mQ, 32 * r, row0, bar_q);
    load_kv(0, 0);
    if (ntiles > 1) load_kv(1, 1);
  }
  bool ok = __syncthreads_and(mbar_wait(bar_q, 0));

  const uint32_t id_s = idesc_tf32(kBM, kBN, false, false);
  const uint32_t id_o = idesc_tf32(kBM, kD, false, true);   // V MN-major
  float m = -INFINITY, l = 0.f;
  float o[kD];
#pragma unroll
  for (int i = 0; i < kD; ++i) o[i] = 0.f;
  // P row of this thread in the swizzled K-major layout: region r (keys 32r..32r+31),
  // row `tid` at 128 B, 16-byte chunk c stored at chunk c ^ (tid & 7).
  unsigned char* prow = sm + kPOff + tid * 128;

  for (int j = 0; j < ntiles && ok; ++j) {
    const int b = j & 1;
    ok = __syncthreads_and(mbar_wait(&bar_kv[b], (uint32_t)(j >> 1) & 1u));
    if (!ok) break;
    tc_fence_after();
    if (tid == 0) {
      const uint64_t qd = sdesc(smem_addr(sm + kQOff), 16, 1024);
      const uint64_t kd = sdesc(smem_addr(sm + kKOff + b * 32768), 16, 1024);
#pragma unroll
      for (int k = 0; k < kD / 8; ++k)
        mma_tf32(t_s, desc_add(qd, kstep_off(k, 16384)), desc_add(kd, kstep_off(k, 16384)), id_s, k > 0);
      mma_commit(bar_s);
    }
    ok = __syncthreads_and(mbar_wait(bar_s, (uint32_t)j & 1u));
    if (!ok) break;
    tc_fence_after();
    // ---- online softmax on this thread's row, 32 columns at a time:
    // pass 1 finds the new row max, pass 2 forms P = exp2(s*scale*log2e - max),
    // its row sum, and writes P into the swizzled K-major tile.
    float mx = m;
#pragma unroll
    for (int c = 0; c < kBN; c += 32) {
      float v[32];
      tmem_ld32(t_s + lane_base + c, v);
#pragma unroll
      for (int i = 0; i < 32; ++i) mx = fmaxf(mx, v[i] * scale_log2);
    }
    const float corr = exp2f(m - mx);
    float sum = 0.f;
#pragma unroll
    for (int c = 0; c < kBN; c += 32) {
      float v[32];
      tmem_ld32(t_s + lane_base + c, v);
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        v[i] = exp2f(fmaf(v[i], scale_log2, -mx));
        sum += v[i];
      }
      unsigned char* region = prow + (c >> 5) * 16384;
#pragma unroll
      for (int q = 0; q < 8; ++q)
        *reinterpret_cast<float4*>(region + ((q ^ (tid & 7)) << 4)) =
            make_float4(round_tf32(v[4 * q]), round_tf32(v[4 * q + 1]), round_tf32(v[4 * q + 2]),
                        round_tf32(v[4 * q + 3]));
    }
    l = l * corr + sum;
    m = mx;
    fence_proxy_async();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (tid == 0) {
      const uint64_t pd = sdesc(smem_addr(sm + kPOff), 16, 1024);
      const uint64_t vd = sdesc_mn(smem_addr(sm + kVOff + b * 32768), 16384);
#pragma unroll
      for (int k = 0; k < kBN / 8; ++k)
        mma_tf32(t_o, desc_add(pd, kstep_off(k, 16384)), desc_add(vd, k * 1024), id_o, k > 0);
      mma_commit(bar_o);
    }
    ok = __syncthreads_and(mbar_wait(bar_o, (uint32_t)j & 1u));
    if (!ok) break;
    tc_fence_after();
    if (tid == 0 && j + 2 < ntiles) load_kv(j + 2, b);
#pragma unroll
    for (int c = 0; c < kD; c += 32) {
      float v[32];
      tmem_ld32(t_o + lane_base + c, v);
#pragma unroll
      for (int i = 0; i < 32; ++i) o[c + i] = fmaf(o[c + i], corr, v[i]);
    }
    tc_fence_before();
    __syncthreads();   // every thread has read S and O_t before the next tile's MMAs overwrite them
    tc_fence_after();
  }
  if (!ok) {
    // record the failure, then give the copies and MMAs already issued a
    // bounded chance to land before the shared and tensor memory go away
    if (tid == 0) fail_timeout();
    mbar_wait(&bar_kv[0], 0, 1 << 16);
    mbar_wait(&bar_kv[1], 0, 1 << 16);
    mbar_wait(bar_s, 0, 1 << 16);
    mbar_wait(bar_o, 0, 1 << 16);
  } else {
    const float inv = 1.f / l;
    float* orow = O + (size_t)(row0 + tid) * kD;
#pragma unroll
    for (int c = 0; c < kD; c += 4)
      *reinterpret_cast<float4*>(orow + c) = make_float4(o[c] * inv, o[c + 1] * inv, o[c + 2] * inv, o[c + 3] * inv);
    if (lse) lse[row0 + tid] = (m + log2f(l)) * 0.69314718055994530942f;  // natural-log units
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, 256);
}

// ------------------------------------------------------------------ two-group kernel, one MMA warp
// 256 query rows per CTA in two groups of 128 (warpgroups 0 and 1, one
// thread per row) that share the K and V tiles.  Warp 8 loads Q and K,
// warp 10 loads V (MN-major), warp 9 alone issues the tensor-core work, in the order
//   S0(0) S1(0) | PV0(0) S0(1) PV1(0) S1(1) | PV0(1) S0(2) PV1(1) S1(2) | ...
// so the next S of one group runs while the other group is in its softmax.
// S_g(j+1) is issued into the columns that hold P_g(j) right after PV_g(j):
// the MMAs of one thread execute in issue order.  Q (rounded, written once
// by the row threads) and P (written back over S, rounded to tf32) are the A
// operands straight from tensor memory, so the products read only K and V
// from shared memory; O accumulates in tensor memory.  The running maximum is raised lazily
// (only when a score exceeds it by more than 2^8), and O is rescaled in place
// then, after that group's previous P V product has completed.  The decision
// is taken per warp, so the warp-collective tensor-memory accesses stay
// convergent.
namespace {
constexpr int kQ3Off = 0;                        // 2 groups x 2 x 16 KB
constexpr int kK3Off = 2 * 32768;                // 2 bufs x K 32 KB
constexpr int kV3Off = kK3Off + 2 * 32768;       // 2 bufs x V 32 KB (dims 0-31, 32-63; MN-major)
constexpr int kBar3Off = kV3Off + 2 * 32768;
constexpr int kSmem3Bytes = kBar3Off + 256 + 1024;
constexpr int kThreads3 = 352;
}  // namespace

__global__ void __launch_bounds__(kThreads3, 1) k_attn_fwd_tc3(const __grid_constant__ CUtensorMap mQ,
                                                              const __grid_constant__ CUtensorMap mK,
                                                              const __grid_constant__ CUtensorMap mV,
                                                              float* __restrict__ O, float* __restrict__ lse, int n,
                                                              float scale_log2) {
  extern __shared__ unsigned char attn3_sm_raw[];
  unsigned char* sm = (unsigned char*)(((uintptr_t)attn3_sm_raw + 1023) & ~(uintptr_t)1023);
  uint64_t* q_full = (uint64_t*)(sm + kBar3Off);
  uint64_t* q_ready = q_full + 1;     // both groups rounded Q (count 256)
  uint64_t* k_full = q_full + 2;      // [2]
  uint64_t* k_empty = q_full + 4;     // [2]
  uint64_t* v_full = q_full + 6;      // [2]
  uint64_t* v_empty = q_full + 8;     // [2]
  uint64_t* s_full = q_full + 10;     // [2] per group: S_g(j) complete
  uint64_t* p_full = q_full + 12;     // [2] per group: P_g(j) written (count 128)
  uint64_t* o_done = q_full + 14;     // [2] per group: P V product j complete
  uint32_t* tslot = (uint32_t*)(sm + kBar3Off + 192);
  volatile int* abort_flag = (volatile int*)(sm + kBar3Off + 196);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int bh = blockIdx.y;
  const int row0 = bh * n + blockIdx.x * 256;
  const int nt = n / kBN;
  if (tid == 0) {
    mbar_init(q_full, 1);
    mbar_init(q_ready, 256);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 128);
      mbar_init(&o_done[i], 1);
    }
    *abort_flag = 0;
    mbar_fence_init();
  }
  __syncthreads();
  if (warp == 0) tmem_alloc(tslot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;   // S_g at g*128, O_g at 256 + g*64, Q_g at 384 + g*64

  if (warp == 8) {
    if (lane == 0) {
      mbar_expect_tx(q_full, 4 * 16384);
      for (int g = 0; g < 2; ++g)
        for (int r = 0; r < 2; ++r) tma_load_2d(sm + kQ3Off + g * 32768 + r * 16384, &mQ, 32 * r, row0 + g * 128, q_full);
      for (int j = 0; j < nt; ++j) {
        const int b = j & 1;
        if (j >= 2 && !mbar_wait(&k_empty[b], (uint32_t)((j - 2) >> 1) & 1u)) { *abort_flag = 1; break; }
        if (*abort_flag) break;
        mbar_expect_tx(&k_full[b], 32768);
        for (int r = 0; r < 2; ++r) tma_load_2d(sm + kK3Off + b * 32768 + r * 16384, &mK, 32 * r, bh * n + j * kBN, &k_full[b]);
      }
    }
  } else if (warp == 10) {
    if (lane == 0) {
      for (int j = 0; j < nt; ++j) {
        const int b = j & 1;
        if (j >= 2 && !mbar_wait(&v_empty[b], (uint32_t)((j - 2) >> 1) & 1u)) { *abort_flag = 1; break; }
        if (*abort_flag) break;
        mbar_expect_tx(&v_full[b], 32768);
        for (int r = 0; r < 2; ++r)
          tma_load_2d(sm + kV3Off + b * 32768 + r * 16384, &mV, 32 * r, bh * n + j * kBN, &v_full[b]);
      }
    }
  } else if (warp == 9) {
    if (lane == 0) {
      const uint32_t id_s = idesc_tf32(kBM, kBN, false, false);
      const uint32_t id_o = idesc_tf32(kBM, kD, false, true);   // V MN-major
      const uint64_t kd = sdesc(smem_addr(sm + kK3Off), 16, 1024);
      // V tiles MN-major: dims 0-31 and 32-63 are two 16 KB blocks of 128 key rows
      const uint64_t vd = sdesc_mn(smem_addr(sm + kV3Off), 16384);
      // S = Q K^T with Q (the A operand) in tensor memory, so only K is read
      // from shared memory
      auto issue_s = [&](int g, int j) {
        const uint64_t kb = desc_add(kd, (j & 1) * 32768);
#pragma unroll
        for (int k = 0; k < kD / 8; ++k)
          mma_tf32_ts(tmem + g * 128, tmem + 384 + g * 64 + k * 8, desc_add(kb, kstep_off(k, 16384)), id_s, k > 0);
        mma_commit(&s_full[g]);
      };
      auto issue_pv = [&](int g, int j) {
        const uint64_t vb = desc_add(vd, (j & 1) * 32768);
        const bool acc0 = j > 0;
#pragma unroll
        for (int k = 0; k < kBN / 8; ++k)
          mma_tf32_ts(tmem + 256 + g * 64, tmem + g * 128 + k * 8, desc_add(vb, k * 1024), id_o,
                      acc0 || k > 0);
        mma_commit(&o_done[g]);
      };
      bool ok = mbar_wait(q_ready, 0) && mbar_wait(&k_full[0], 0);
      if (ok) {
        tc_fence_after();
        issue_s(0, 0);
        issue_s(1, 0);
        mma_commit(&k_empty[0]);
      }
      for (int j = 0; j < nt && ok; ++j) {
        const int b = j & 1;
        const bool more = j + 1 < nt;
        if (!mbar_wait(&v_full[b], (uint32_t)(j >> 1) & 1u) || !mbar_wait(&p_full[0], (uint32_t)j & 1u)) { ok = false; break; }
        tc_fence_after();
        issue_pv(0, j);
        if (more) {
          if (!mbar_wait(&k_full[b ^ 1], (uint32_t)((j + 1) >> 1) & 1u)) { ok = false; break; }
          tc_fence_after();
          issue_s(0, j + 1);
        }
        if (!mbar_wait(&p_full[1], (uint32_t)j & 1u)) { ok = false; break; }
        tc_fence_after();
        issue_pv(1, j);
        mma_commit(&v_empty[b]);
        if (more) {
          issue_s(1, j + 1);
          mma_commit(&k_empty[b ^ 1]);
        }
      }
      if (!ok) *abort_flag = 1;
    }
  } else if (warp < 8) {
    // ---------------- softmax group g, one thread per query row
    const int g = warp >> 2, t = tid & 127;
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
    const uint32_t t_s = tmem + g * 128 + lane_base, t_o = tmem + 256 + g * 64 + lane_base;
    bool ok = mbar_wait(q_full, 0);
    if (!ok) *abort_flag = 1;
    {
      // this thread's Q row, rounded to the nearest tf32, into its tensor-memory
      // lane: columns 0-63 of Q_g (the staged row is 128-byte swizzled: logical
      // 16-byte chunk c of row t sits at chunk c ^ (t & 7))
      const unsigned char* qrow = sm + kQ3Off + g * 32768 + t * 128;
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        float v[32];
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const float4 x = *reinterpret_cast<const float4*>(qrow + r * 16384 + ((c ^ (t & 7)) << 4));
          v[4 * c] = round_tf32(x.x);
          v[4 * c + 1] = round_tf32(x.y);
          v[4 * c + 2] = round_tf32(x.z);
          v[4 * c + 3] = round_tf32(x.w);
        }
        tmem_st32(tmem + 384 + g * 64 + lane_base + 32 * r, v);
      }
      tmem_st_wait();
      tc_fence_before();
    }
    mbar_arrive(q_ready);
    // m: the exponent offset in use (log2 units), raised only when a score
    // exceeds it by more than 8, so p = 2^(s*c - m) <= 256
    float m = -INFINITY, l = 0.f;
    for (int j = 0; j < nt; ++j) {
      ok = named_bar_and(1 + g, 128, ok && mbar_wait(&s_full[g], (uint32_t)j & 1u) && !*abort_flag);
      if (!ok) break;
      tc_fence_after();
      uint32_t sr[4][32];
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld32_nowait(t_s + 32 * c, sr[c]);
      tmem_ld_wait();
      // row max and row sum over 8 independent partials: a single chain of
      // 128 dependent operations per thread left the few softmax warps idle
      float mx8[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) mx8[k] = -INFINITY;
#pragma unroll
      for (int c = 0; c < 4; ++c)
#pragma unroll
        for (int i = 0; i < 32; ++i) mx8[i & 7] = fmaxf(mx8[i & 7], __uint_as_float(sr[c][i]));
      const float mraw = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                               fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7])));
      const float mt = mraw * scale_log2;
      const bool up = mt > m + 8.f;
      if (__any_sync(0xffffffffu, up)) {
        const float corr = up ? ex2_approx(m - mt) : 1.f;   // 0 on the first tile
        if (up) {
          l *= corr;
          m = mt;
        }
        if (j > 0) {
          // O of this group may still be written by P V product j-1
          if (!__all_sync(0xffffffffu, mbar_wait(&o_done[g], (uint32_t)(j - 1) & 1u))) *abort_flag = 1;
          tc_fence_after();
#pragma unroll 1
          for (int c = 0; c < kD; c += 16) {
            float v[16];
            tmem_ld16(t_o + c, v);
#pragma unroll
            for (int i = 0; i < 16; ++i) v[i] *= corr;
            tmem_st16(t_o + c, v);
          }
        }
      }
      float sm8[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) sm8[k] = 0.f;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        float v[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const float p = ex2_approx(fmaf(__uint_as_float(sr[c][i]), scale_log2, -m));
          sm8[i & 7] += p;
          v[i] = round_tf32_int(p);
        }
        tmem_st32(t_s + 32 * c, v);
      }
      tmem_st_wait();
      l += ((sm8[0] + sm8[1]) + (sm8[2] + sm8[3])) + ((sm8[4] + sm8[5]) + (sm8[6] + sm8[7]));
      tc_fence_before();
      mbar_arrive(&p_full[g]);
    }
    if (ok) ok = named_bar_and(1 + g, 128, mbar_wait(&o_done[g], (uint32_t)(nt - 1) & 1u) && !*abort_flag);
    if (ok) {
      tc_fence_after();
      const float inv = 1.f / l;
      float* orow = O + (size_t)(row0 + g * 128 + t) * kD;
#pragma unroll
      for (int c = 0; c < kD; c += 32) {
        float v[32];
        tmem_ld32(t_o + c, v);
#pragma unroll
        for (int i = 0; i < 32; i += 4)
          *reinterpret_cast<float4*>(orow + c + i) = make_float4(v[i] * inv, v[i + 1] * inv, v[i + 2] * inv, v[i + 3] * inv);
      }
      if (lse) lse[row0 + g * 128 + t] = (m + log2f(l)) * 0.69314718055994530942f;
    } else if (t == 0) {
      *abort_flag = 1;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (*abort_flag) {
    if (tid == 0) fail_timeout();
    // bounded drain of anything still in flight before the memory is released
    mbar_wait(q_full, 0, 1 << 14);
    for (int i = 0; i < 2; ++i) {
      mbar_wait(&k_full[i], 0, 1 << 14);
      mbar_wait(&v_full[i], 0, 1 << 14);
      mbar_wait(&s_full[i], 0, 1 << 14);
      mbar_wait(&o_done[i], 0, 1 << 14);
    }
  }
  if (warp == 0) tmem_dealloc(tmem, 512);
}

// K and V -> copies rounded to the nearest tf32 (the tensor core would
// truncate), in one pass over both.
__global__ void k_round_tf32_2(const float4* __restrict__ K, const float4* __restrict__ V, float4* __restrict__ Kr,
                               float4* __restrict__ Vr, long long n4) {
  long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (; i < n4; i += stride) {
    const float4 k = K[i], v = V[i];
    Kr[i] = make_float4(round_tf32_int(k.x), round_tf32_int(k.y), round_tf32_int(k.z), round_tf32_int(k.w));
    Vr[i] = make_float4(round_tf32_int(v.x), round_tf32_int(v.y), round_tf32_int(v.z), round_tf32_int(v.w));
  }
}

// Per-device scratch for the rounded K and V, grown on demand and kept (it is reused by every call
// on that device; calls on one device are stream-ordered by the caller).
static int vt_scratch(size_t bytes, void** out) {
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

int attention_fwd_tc(const float* Q, const float* K, const float* V, float* O, float* lse, long long blocks, int n,
                     int dk, int dv, float scale, cudaStream_t s, bool* handled) {
  *handled = false;
  if (dk != kD || dv != kD || n < kBN || (n % kBN) != 0 || blocks <= 0 || blocks > 65535) return AMC_OK;
  if (((uintptr_t)Q | (uintptr_t)K | (uintptr_t)V | (uintptr_t)O) & 15) return AMC_OK;
  const uint64_t rows = (uint64_t)blocks * n;
  if (rows > 0x7fffffffull) return AMC_OK;
  *handled = true;
  float* Kr = nullptr;
  const size_t tbytes = (size_t)rows * kD * sizeof(float);
  int rc0 = vt_scratch(2 * tbytes, (void**)&Kr);
  if (rc0) return rc0;
  float* Vr = Kr + (size_t)rows * kD;
  k_round_tf32_2<<<(unsigned)(num_sms() * 8), 256, 0, s>>>((const float4*)K, (const float4*)V, (float4*)Kr, (float4*)Vr,
                                                          (long long)(rows * kD / 4));
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "k_round_tf32_2");
  // K tiles K-major (128-byte swizzle); V tiles MN-major (128-byte swizzle in
  // 32-byte atoms): the P V product contracts over keys, the rows of V
  CUtensorMap mQ, mK, mV;
  int rc = make_tmap_2d_f32(&mQ, Q, rows, kD, kD, 128);
  if (!rc) rc = make_tmap_2d_f32(&mK, Kr, rows, kD, kD, 128);
  if (!rc) rc = make_tmap_2d_f32_swz(&mV, Vr, rows, kD, kD, 32, 128, TmapSwizzle::k128Atom32);
  if (rc) return rc;
  const float scale_log2 = scale * 1.4426950408889634f;
  static std::atomic<uint64_t> attr3{0}, attr1{0};
  if (n % 256 == 0) {
    int rca = smem_attr_once(k_attn_fwd_tc3, kSmem3Bytes, attr3);
    if (rca) return rca;
    k_attn_fwd_tc3<<<dim3(n / 256, (unsigned)blocks), kThreads3, kSmem3Bytes, s>>>(mQ, mK, mV, O, lse, n, scale_log2);
  } else {
    int rca = smem_attr_once(k_attn_fwd_tc, kSmemBytes, attr1);
    if (rca) return rca;
    k_attn_fwd_tc<<<dim3(n / kBM, (unsigned)blocks), 128, kSmemBytes, s>>>(mQ, mK, mV, O, lse, n, scale_log2);
  }
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "k_attn_fwd_tc");
  return AMC_OK;
}

int attention_check_error() {
  int e = 0;
  AMC_CUDA(cudaMemcpyFromSymbol(&e, g_attn_error, sizeof(int)));
  if (e) {
    int z = 0;
    AMC_CUDA(cudaMemcpyToSymbol(g_attn_error, &z, sizeof(int)));
    return fail(e, "attention: a bounded wait on the tensor-core pipeline gave up");
  }
  return AMC_OK;
}

}  // namespace amc
