// Tensor-core 3x3 convolution (stride 1, pad 1, 64 -> 64 channels, NCHW),
// tcgen05 kind::tf32 implicit GEMM; used by the forward and the data-gradient
// (a forward convolution of dY with the flipped, transposed weights).
//
// The reference forms im2col(X) explicitly and multiplies it by the
// flattened weights per image (execute-conv2d-blas, realization.scm:166-252).
// Here no column matrix exists:
//   - an output tile is 2 output rows x 64 columns (128 positions = MMA M).
//     Four producer warps read the 4 input rows it needs straight from NCHW
//     (64 positions per row from column -1, zero outside the image, rounded
//     to the nearest tf32) and write each position's 32 channels as a
//     128-byte row of a K-major, 128-byte-swizzled tile (two tiles: channels
//     0-31 and 32-63); no padded copy of the input exists;
//   - tap (kh, kw) of the tile is the same shared tile read from position
//     kh*64 + kw on: its A descriptor starts (kh*64 + kw) * 128 bytes in, so
//     all 9 taps are address offsets of one staged tile;
//   - B is the tap's (64 out x 64 in) weight block, K-major, resident in
//     shared memory for the whole kernel;
//   - 72 MMAs (9 taps x 64 channels / 8) accumulate one 128 x 64 f32 tile in
//     tensor memory, issued by two warps (one per 32-channel chunk, 36 each,
//     into separate accumulators the epilogue adds): one issuing thread
//     cannot keep the tensor pipe fed with N=64 products.  Two accumulator
//     pairs alternate so the epilogue of one tile overlaps the MMAs of the
//     next.
// Output columns 56..63 of a tile are computed on zero padding and dropped.
// Warp roles: warps 0-3 input producers, 4-7 epilogue, 8 weight loads (TMA), 9-10 MMA issuers.
#include <cudaTypedefs.h>

#include "amc_internal.h"
#include "amc_tc.cuh"

namespace amc {

struct ConvShape {
  int N, C, H, W, K, KH, KW, SH, SW, PH, PW, OH, OW;
};

using namespace tc;

namespace {

constexpr int kC = 64;                    // in = out channels
constexpr int kPosRow = 64;               // positions per staged input row
constexpr int kRegion = 4 * kPosRow * 128 + 1024;   // 4 input rows + slack (1024-aligned)
constexpr int kWOff = 0;                  // 9 taps x 2 chunks x 8 KB
constexpr int kXOff = kWOff + 9 * 2 * 8192;         // 2 chunk regions
constexpr int kBarOffC = kXOff + 2 * kRegion;
constexpr int kConvSmem = kBarOffC + 256 + 1024;
constexpr int kConvThreads = 352;   // warps 0-3 input producers, 4-7 epilogue, 8 weights, 9-10 MMA

__device__ int g_conv_error;

}  // namespace

__global__ void __launch_bounds__(kConvThreads, 1) k_conv3x3_tc(const float* __restrict__ X,
                                                               const __grid_constant__ CUtensorMap mW,
                                                               float* __restrict__ Y, int N, int H, int Wd) {
  extern __shared__ unsigned char conv_sm_raw[];
  unsigned char* sm = (unsigned char*)(((uintptr_t)conv_sm_raw + 1023) & ~(uintptr_t)1023);
  uint64_t* x_full = (uint64_t*)(sm + kBarOffC);   // [2] per channel chunk (128 producer arrivals)
  uint64_t* x_empty = x_full + 2;     // [2]
  uint64_t* acc_full = x_full + 4;    // [2] per accumulator
  uint64_t* acc_empty = x_full + 6;   // [2]
  uint64_t* w_full = x_full + 8;      // [9] per tap: both channel chunks of its weights
  uint32_t* tslot = (uint32_t*)(sm + kBarOffC + 192);
  volatile int* abort_flag = (volatile int*)(sm + kBarOffC + 196);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int pairs = H / 2;
  const int ntiles = N * pairs;
  if (tid == 0) {
    for (int t = 0; t < 9; ++t) mbar_init(&w_full[t], 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&x_full[i], 128);
      mbar_init(&x_empty[i], 1);
      mbar_init(&acc_full[i], 2);   // one commit from each chunk's MMA warp
      mbar_init(&acc_empty[i], 1);
    }
    *abort_flag = 0;
    mbar_fence_init();
  }
  __syncthreads();
  if (warp == 0) tmem_alloc(tslot, 256);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;

  if (warp < 4) {
    // ---- producers: the tile's 4 input rows (oh0-1 .. oh0+2) x 64 positions
    // (columns -1 .. 62) x 32 channels per chunk, zero outside the image,
    // rounded to tf32, written as K-major 128-byte rows (position q at q*128,
    // logical 16-byte chunk j of a row at j ^ (q & 7)).  Warp w takes the
    // (row, channel-quad) pairs 8w .. 8w+7; each lane one position per half.
    // The next chunk's values are loaded into registers before the wait for
    // its buffer, so the global-load latency overlaps the products.
    const size_t plane = (size_t)H * Wd;
    float4 buf[16];
    auto fetch = [&](int tile, int c) {
      const int n = tile / pairs, oh0 = (tile % pairs) * 2;
#pragma unroll
      for (int pi = 0; pi < 8; ++pi) {
        const int pr = warp * 8 + pi, r = pr >> 3, j = pr & 7;
        const int ih = oh0 - 1 + r;
        const bool rowok = ih >= 0 && ih < H;
        const float* src = X + ((size_t)n * kC + 32 * c + 4 * j) * plane + (size_t)(rowok ? ih : 0) * Wd;
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          const int iw = lane + 32 * half - 1;
          float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
          if (rowok && iw >= 0 && iw < Wd) {
            v.x = __ldg(src + iw);
            v.y = __ldg(src + plane + iw);
            v.z = __ldg(src + 2 * plane + iw);
            v.w = __ldg(src + 3 * plane + iw);
          }
          buf[pi * 2 + half] = v;
        }
      }
    };
    int li = 0, tile = blockIdx.x;
    if (tile < ntiles) fetch(tile, 0);
    for (; tile < ntiles; tile += gridDim.x, ++li) {
      for (int c = 0; c < 2; ++c) {
        if (li > 0 && !mbar_wait(&x_empty[c], (uint32_t)(li - 1) & 1u)) *abort_flag = 1;
        if (*abort_flag) break;
        unsigned char* region = sm + kXOff + c * kRegion;
#pragma unroll
        for (int pi = 0; pi < 8; ++pi) {
          const int pr = warp * 8 + pi, r = pr >> 3, j = pr & 7;
#pragma unroll
          for (int half = 0; half < 2; ++half) {
            const int q = r * kPosRow + lane + 32 * half;
            const float4 v = buf[pi * 2 + half];
            *reinterpret_cast<float4*>(region + q * 128 + ((j ^ (q & 7)) << 4)) =
                make_float4(round_tf32(v.x), round_tf32(v.y), round_tf32(v.z), round_tf32(v.w));
          }
        }
        fence_proxy_async();
        mbar_arrive(&x_full[c]);
        // next chunk: chunk 1 of this tile, or chunk 0 of the next tile
        if (c == 0) fetch(tile, 1);
        else if (tile + (int)gridDim.x < ntiles) fetch(tile + gridDim.x, 0);
      }
      if (*abort_flag) break;
    }
  } else if (warp == 8) {
    if (lane == 0) {
      // the weights once, tap by tap (boxes of 32 in-channels x 64 out-channels)
      for (int t = 0; t < 9; ++t) {
        mbar_expect_tx(&w_full[t], 2 * 8192);
        for (int c = 0; c < 2; ++c) tma_load_2d(sm + kWOff + (2 * t + c) * 8192, &mW, 0, (2 * t + c) * 64, &w_full[t]);
      }
    }
  } else if (warp == 9 || warp == 10) {
    // warp 9 + c issues the products of input-channel chunk c into its own
    // accumulator (tensor memory a * 128 + c * 64); the epilogue adds the two
    if (lane == 0) {
      const int c = warp - 9;
      const uint32_t idesc = idesc_tf32(128, kC, false, false);
      const uint64_t xd = sdesc(smem_addr(sm + kXOff + c * kRegion), 16, 1024);
      const uint64_t wd = sdesc(smem_addr(sm + kWOff + c * 8192), 16, 1024);
      bool ok = true;
      int li = 0;
      for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x, ++li) {
        const int a = li & 1;
        if (li >= 2 && !mbar_wait(&acc_empty[a], (uint32_t)((li - 2) >> 1) & 1u)) { ok = false; break; }
        if (!mbar_wait(&x_full[c], (uint32_t)li & 1u)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d = tmem + a * 2 * kC + c * kC;
#pragma unroll
        for (int tap = 0; tap < 9; ++tap) {
          const int kh = tap / 3, kw = tap % 3;
          if (li == 0) {
            if (!mbar_wait(&w_full[tap], 0)) ok = false;
            tc_fence_after();
          }
#pragma unroll
          for (int k = 0; k < 4; ++k)
            mma_tf32(d, desc_add(xd, (kh * kPosRow + kw) * 128 + k * 32), desc_add(wd, tap * 2 * 8192 + k * 32), idesc,
                     (tap | k) != 0);
        }
        mma_commit(&x_empty[c]);
        mma_commit(&acc_full[a]);
        if (*abort_flag) break;
      }
      if (!ok) *abort_flag = 1;
    }
  } else if (warp >= 4 && warp < 8) {
    // epilogue warpgroup: TMEM lane q = output position q of the tile
    const int q = tid - 128;
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
    const int r = q / kPosRow, col = q % kPosRow;
    int li = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++li) {
      const int a = li & 1;
      ok = named_bar_and(1, 128, mbar_wait(&acc_full[a], (uint32_t)(li >> 1) & 1u) && !*abort_flag);
      if (!ok) break;
      tc_fence_after();
      // 16 output channels at a time: the two chunk accumulators added and
      // stored at once (measured faster than holding all 64 and storing them
      // in one burst after the release)
      const int n = tile / pairs, oh = (tile % pairs) * 2 + r;
      float* yp = Y + ((size_t)n * kC * H + oh) * Wd + col;
#pragma unroll 1
      for (int h = 0; h < 4; ++h) {
        float v[16], u[16];
        tmem_ld16(tmem + a * 2 * kC + lane_base + 16 * h, v);
        tmem_ld16(tmem + a * 2 * kC + kC + lane_base + 16 * h, u);
        if (col < Wd) {
#pragma unroll
          for (int i = 0; i < 16; ++i) __stcs(yp + (size_t)(16 * h + i) * H * Wd, v[i] + u[i]);
        }
      }
      tc_fence_before();
      named_bar(1, 128);
      if (q == 0) mbar_arrive(&acc_empty[a]);
    }
    if (!ok && q == 0) atomicExch(&g_conv_error, AMC_ERR_TIMEOUT);
  }
  tc_fence_before();
  __syncthreads();
  if (*abort_flag) {
    for (int i = 0; i < 2; ++i) mbar_wait(&acc_full[i], 0, 1 << 14);
    for (int t = 0; t < 9; ++t) mbar_wait(&w_full[t], 0, 1 << 14);
  }
  if (warp == 0) tmem_dealloc(tmem, 256);
}

// Weights (64 out, 64 in, 3, 3) -> [tap][in-chunk][out][32 in], rounded to tf32.
// flip != 0 gives the data-gradient weights W'[in][out][2-kh][2-kw].
__global__ void k_conv_weights(const float* __restrict__ W, float* __restrict__ Wt, int flip) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= 9 * kC * kC) return;
  const int ci = i % 32, co = (i / 32) % kC, chunk = (i / (32 * kC)) % 2, tap = i / (2 * 32 * kC);
  const int kh = tap / 3, kw = tap % 3, cin = chunk * 32 + ci;
  const float v = flip ? W[(((size_t)cin * kC + co) * 3 + (2 - kh)) * 3 + (2 - kw)]
                       : W[(((size_t)co * kC + cin) * 3 + kh) * 3 + kw];
  Wt[i] = round_tf32(v);
}

static int conv_scratch(size_t bytes, void** out) {
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

static bool conv_tc_shape(const ConvShape& s) {
  return s.C == kC && s.K == kC && s.KH == 3 && s.KW == 3 && s.SH == 1 && s.SW == 1 && s.PH == 1 && s.PW == 1 &&
         s.H % 2 == 0 && s.W + 2 <= kPosRow && s.W % 4 == 0 && s.W >= 8 && s.N >= 1 &&
         (size_t)s.N * (s.H + 2) < (1u << 31);
}

static int conv_run(const float* in, const float* W, float* out, const ConvShape& s, int flip, cudaStream_t st) {
  void* scratch = nullptr;
  int rc = conv_scratch(9 * kC * kC * sizeof(float) + 1024, &scratch);
  if (rc) return rc;
  float* Wt = (float*)(((uintptr_t)scratch + 1023) & ~(uintptr_t)1023);
  k_conv_weights<<<(9 * kC * kC + 255) / 256, 256, 0, st>>>(W, Wt, flip);
  AMC_CUDA(cudaGetLastError());
  CUtensorMap mW;
  rc = make_tmap_2d_f32(&mW, Wt, 9 * 2 * kC, 32, 32, 64);
  if (rc) return rc;
  static std::atomic<uint64_t> attr{0};
  rc = smem_attr_once(k_conv3x3_tc, kConvSmem, attr);
  if (rc) return rc;
  const int ntiles = s.N * (s.H / 2);
  const int grid = ntiles < num_sms() ? ntiles : num_sms();
  k_conv3x3_tc<<<grid, kConvThreads, kConvSmem, st>>>(in, mW, out, s.N, s.H, s.W);
  AMC_CUDA(cudaGetLastError());
  return AMC_OK;
}

int conv_fwd_tc(const float* X, const float* W, float* Y, const ConvShape& s, cudaStream_t st, bool* handled) {
  *handled = conv_tc_shape(s);
  if (!*handled) return AMC_OK;
  return conv_run(X, W, Y, s, 0, st);
}

int conv_dgrad_tc(const float* dY, const float* W, float* dX, const ConvShape& s, cudaStream_t st, bool* handled) {
  *handled = conv_tc_shape(s);
  if (!*handled) return AMC_OK;
  return conv_run(dY, W, dX, s, 1, st);
}

// ------------------------------------------------------------------ weight gradient
// dW[co, ci, kh, kw] = sum_{n, q} dY[n, co, q - (kh-1)*W] * X_kw[n, ci, q]
// over flattened positions q of the H x W plane, where X_kw[q] = X[q + kw - 1]
// with zeros where column w + kw - 1 leaves the row.  The reference's order is
// a batch sum of per-image GEMMs dY_n . im2col(X_n)^T; here the position sum
// is split across CTAs and the CTA partials are added in a fixed order by a
// second kernel.
// Positions are the K dimension, so the NCHW planes are already K-major and
// the kernel reads dY and X as they are:
//   - per K-chunk of 32 positions the TMA warp loads A = dY rows for kh = 0,
//     1, 2 (row shifts of W positions are TMA coordinate offsets, zero-filled
//     outside the plane), B1 = X (kw = 1) and two 4-column halo boxes of X;
//   - warps 4-7 write A, rounded to the nearest tf32, into tensor memory
//     (the products' A operand, read there by all three column taps instead
//     of three times from shared memory), round B1 in place and write the
//     column-shifted B0 and B2 (a 4-byte shift cannot start a descriptor);
//   - warp 1 + kw issues the two M=128 products of column tap kw: kh rows
//     (0,1) and (1,2); their 64-column accumulators stay in tensor memory
//     for the CTA's whole chunk range.
namespace {
constexpr int kWgBlk = 8192;                       // 64 rows x 128 B, K-major, 128-byte swizzle
constexpr int kWgHalo = 64 * 16;                   // 64 rows x 4 floats, row-major
constexpr int kWgHaloOff = 6 * kWgBlk;             // left halo, then right halo
constexpr int kWgStage = 6 * kWgBlk + 2 * kWgHalo; // A0-2, B0-2, halos: 50 KB
constexpr int kWgStages = 4;
constexpr int kWgBarOff = kWgStages * kWgStage;
constexpr int kWgSmem = kWgBarOff + 256 + 1024;
constexpr int kWgPart = 3 * 2 * 128 * kC;          // floats of one CTA's partial: [kw][block][lane][64]
static_assert(kWgStage % 1024 == 0, "stages stay 1024-byte aligned");
static_assert(kWgSmem <= 232448, "weight-gradient shared memory");

__device__ __forceinline__ float4 round4(float4 v) {
  return make_float4(round_tf32(v.x), round_tf32(v.y), round_tf32(v.z), round_tf32(v.w));
}
}  // namespace

__global__ void __launch_bounds__(256, 1) k_conv_wgrad_tc(const __grid_constant__ CUtensorMap mDY,
                                                         const __grid_constant__ CUtensorMap mX,
                                                         const __grid_constant__ CUtensorMap mXh,
                                                         float* __restrict__ partials, int N, int HW,
                                                         int Wd, int chunks_per_img) {
  extern __shared__ unsigned char wg_sm_raw[];
  unsigned char* sm = (unsigned char*)(((uintptr_t)wg_sm_raw + 1023) & ~(uintptr_t)1023);
  uint64_t* full = (uint64_t*)(sm + kWgBarOff);   // [kWgStages] TMA landed
  uint64_t* ready = full + kWgStages;             // [kWgStages] rounded and shifted
  uint64_t* empty = full + 2 * kWgStages;         // [kWgStages] products done
  uint64_t* done = full + 3 * kWgStages;
  uint64_t* tfree = done + 1;                     // [2] products read tensor-memory A buffer
  uint32_t* tslot = (uint32_t*)(sm + kWgBarOff + 192);
  volatile int* abort_flag = (volatile int*)(sm + kWgBarOff + 196);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int total = N * chunks_per_img;
  const int c0 = (int)((long long)total * blockIdx.x / gridDim.x);
  const int c1 = (int)((long long)total * (blockIdx.x + 1) / gridDim.x);
  if (tid == 0) {
    for (int i = 0; i < kWgStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&ready[i], 128);
      mbar_init(&empty[i], 3);   // one commit from each column tap's MMA warp
    }
    mbar_init(done, 3);
    for (int i = 0; i < 2; ++i) mbar_init(&tfree[i], 3);
    *abort_flag = 0;
    mbar_fence_init();
  }
  __syncthreads();
  if (warp == 0) tmem_alloc(tslot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;
  // accumulators at kw * 128 + blk * 64 (0..383); the A operands (dY rows,
  // blocks kh (0,1) and (1,2), 32 positions each) at 384 + b * 64 + blk * 32
  // for buffer b = chunk & 1
  const uint32_t t_a = tmem + 384;
  if (warp == 0) {
    if (lane == 0) {
      for (int c = c0, it = 0; c < c1; ++c, ++it) {
        const int st = it % kWgStages;
        if (it >= kWgStages && !mbar_wait(&empty[st], (uint32_t)((it / kWgStages) - 1) & 1u)) { *abort_flag = 1; break; }
        if (*abort_flag) break;
        const int n = c / chunks_per_img, q0 = (c % chunks_per_img) * 32;
        unsigned char* sb = sm + st * kWgStage;
        mbar_expect_tx(&full[st], 4 * kWgBlk + 2 * kWgHalo);
        for (int kh = 0; kh < 3; ++kh) tma_load_2d(sb + kh * kWgBlk, &mDY, q0 - (kh - 1) * Wd, n * kC, &full[st]);
        tma_load_2d(sb + 4 * kWgBlk, &mX, q0, n * kC, &full[st]);
        tma_load_2d(sb + kWgHaloOff, &mXh, q0 - 4, n * kC, &full[st]);
        tma_load_2d(sb + kWgHaloOff + kWgHalo, &mXh, q0 + 32, n * kC, &full[st]);
      }
    }
  } else if (warp >= 1 && warp <= 3) {
    // warp 1 + kw issues the two products of column tap kw (its own accumulators)
    if (lane == 0) {
      const int kw = warp - 1;
      const uint32_t idesc = idesc_tf32(128, kC, false, false);
      const uint64_t sdesc0 = sdesc(smem_addr(sm), 16, 1024);
      bool ok = true;
      for (int c = c0, it = 0; c < c1; ++c, ++it) {
        const int st = it % kWgStages;
        if (!mbar_wait(&ready[st], (uint32_t)(it / kWgStages) & 1u)) { ok = false; break; }
        tc_fence_after();
        const uint64_t sd = desc_add(sdesc0, st * kWgStage);
        const uint32_t ta = t_a + (uint32_t)((it & 1) * 64);
        const bool acc0 = it > 0;
#pragma unroll
        for (int k = 0; k < 4; ++k)
#pragma unroll
          for (int blk = 0; blk < 2; ++blk)
            mma_tf32_ts(tmem + (uint32_t)(kw * 128 + blk * 64), ta + blk * 32 + k * 8,
                        desc_add(sd, (3 + kw) * kWgBlk + k * 32), idesc, acc0 || k > 0);
        mma_commit(&empty[st]);
        mma_commit(&tfree[it & 1]);
        if (*abort_flag) break;
      }
      if (!ok) *abort_flag = 1;
      mma_commit(done);
    }
  } else if (warp >= 4) {
    // ---- operand preparation: thread t owns row r (a channel) and positions
    // 16h..16h+15 of every block; logical 16-byte chunk j of row r sits at
    // chunk j ^ (r & 7) (the 128-byte swizzle)
    const int t = tid - 128, r = t >> 1, h = t & 1;
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
    bool okp = true;
    for (int c = c0, it = 0; c < c1 && okp; ++c, ++it) {
      const int st = it % kWgStages;
      if (!mbar_wait(&full[st], (uint32_t)(it / kWgStages) & 1u) ||
          (it >= 2 && !mbar_wait(&tfree[it & 1], (uint32_t)((it - 2) >> 1) & 1u)) || *abort_flag) {
        *abort_flag = 1;
        okp = false;
        break;
      }
      unsigned char* sb = sm + st * kWgStage;
      // A into tensor memory: lane t of block blk holds dY row (t & 63) of
      // row shift kh = blk + (t >> 6), its 32 positions rounded
      {
        const int ar = t & 63, asw = ar & 7;
#pragma unroll
        for (int blk = 0; blk < 2; ++blk) {
          const unsigned char* arow = sb + (blk + (t >> 6)) * kWgBlk + ar * 128;
          float v[32];
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const float4 x4 = *reinterpret_cast<const float4*>(arow + ((i ^ asw) << 4));
            v[4 * i] = round_tf32(x4.x);
            v[4 * i + 1] = round_tf32(x4.y);
            v[4 * i + 2] = round_tf32(x4.z);
            v[4 * i + 3] = round_tf32(x4.w);
          }
          tmem_st32(t_a + (uint32_t)((it & 1) * 64 + blk * 32) + lane_base, v);
        }
      }
      unsigned char* row = sb + r * 128;
      const int sw = r & 7;
      float x[16];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float4 v = *reinterpret_cast<const float4*>(row + 4 * kWgBlk + (((4 * h + i) ^ sw) << 4));
        x[4 * i] = v.x; x[4 * i + 1] = v.y; x[4 * i + 2] = v.z; x[4 * i + 3] = v.w;
      }
      // neighbours: position 16h - 1 and 16h + 16 of this row (a halo column
      // at the chunk ends; re-reading a neighbour already rounded is harmless)
      const float* halo = reinterpret_cast<const float*>(sb + kWgHaloOff);
      const float left = h ? *reinterpret_cast<const float*>(row + 4 * kWgBlk + ((3 ^ sw) << 4) + 12)
                           : halo[r * 4 + 3];
      const float right = h ? halo[kWgHalo / 4 + r * 4]
                            : *reinterpret_cast<const float*>(row + 4 * kWgBlk + ((4 ^ sw) << 4));
      const int q = (c % chunks_per_img) * 32 + 16 * h;
      int w = q % Wd;
      float b0[16], b2[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const float xm = j == 0 ? left : x[j - 1];
        const float xp = j == 15 ? right : x[j + 1];
        b0[j] = w == 0 ? 0.f : round_tf32(xm);
        b2[j] = w == Wd - 1 ? 0.f : round_tf32(xp);
        w = w + 1 == Wd ? 0 : w + 1;
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int off = ((4 * h + i) ^ sw) << 4;
        *reinterpret_cast<float4*>(row + 3 * kWgBlk + off) = make_float4(b0[4 * i], b0[4 * i + 1], b0[4 * i + 2], b0[4 * i + 3]);
        *reinterpret_cast<float4*>(row + 4 * kWgBlk + off) =
            round4(make_float4(x[4 * i], x[4 * i + 1], x[4 * i + 2], x[4 * i + 3]));
        *reinterpret_cast<float4*>(row + 5 * kWgBlk + off) = make_float4(b2[4 * i], b2[4 * i + 1], b2[4 * i + 2], b2[4 * i + 3]);
      }
      tmem_st_wait();
      tc_fence_before();
      fence_proxy_async();
      mbar_arrive(&ready[st]);
    }
    // ---- epilogue: TMEM lane = row
    const bool ok = named_bar_and(1, 128, mbar_wait(done, 0) && !*abort_flag);
    if (ok && c1 > c0) {
      tc_fence_after();
      // lanes 0-63 of block 0 are kh=0, 64-127 kh=1; block 1 lanes 64-127 are
      // kh=2.  Partials keep the tensor-memory layout [kw][block][lane][64],
      // so each thread writes its row's 64 values contiguously.
      const int lr = tid - 128;
      float* part = partials + (size_t)blockIdx.x * kWgPart;
      for (int kw = 0; kw < 3; ++kw)
        for (int blk = 0; blk < 2; ++blk) {
          if (blk == 1 && lr < 64) continue;   // duplicate of kh=1 (whole warps 4 and 5)
          float4* dst = reinterpret_cast<float4*>(part + ((size_t)(kw * 2 + blk) * 128 + lr) * kC);
          for (int half = 0; half < 2; ++half) {
            float v[32];
            tmem_ld32(tmem + (uint32_t)(kw * 128 + blk * 64 + half * 32) + lane_base, v);
#pragma unroll
            for (int i = 0; i < 8; ++i) dst[half * 8 + i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
          }
        }
    } else if (!ok && tid == 128) {
      atomicExch(&g_conv_error, AMC_ERR_TIMEOUT);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (*abort_flag) {
    for (int i = 0; i < kWgStages; ++i) mbar_wait(&full[i], 0, 1 << 14);
    mbar_wait(done, 0, 1 << 14);
    for (int i = 0; i < 2; ++i) mbar_wait(&tfree[i], 0, 1 << 14);
  }
  if (warp == 0) tmem_dealloc(tmem, 512);
}

// dW = sum of the CTA partials in a fixed order (CTAs without chunks add
// nothing).  A block takes 32 outputs (consecutive in-channels of one
// (kw, kh, out-channel)) and 8 groups of partials: group g adds partials
// g, g+8, ... in ascending order, then the 8 group sums are added in index
// order, so the result does not depend on timing.
__global__ void __launch_bounds__(256) k_wgrad_reduce(const float* __restrict__ partials, float* __restrict__ dW,
                                                      int nparts, const int* counts) {
  __shared__ float red[8][33];
  const int l = threadIdx.x & 31, g = threadIdx.x >> 5;
  const int o = blockIdx.x * 32 + l;   // (kw, kh, co, ci), ci fastest
  const int ci = o & 63, co = (o >> 6) & 63, kh = (o >> 12) % 3, kw = (o >> 12) / 3;
  const int blk = kh == 2 ? 1 : 0, lane = kh == 2 ? 64 + co : kh * 64 + co;
  const size_t off = ((size_t)(kw * 2 + blk) * 128 + lane) * kC + ci;
  // the partials of group g are added in ascending order; the loads of four
  // of them are issued together (a partial of a CTA that had no chunk is
  // read but not added)
  float s = 0.f;
  int p = g;
  for (; p + 24 < nparts; p += 32) {
    const int c0 = counts[p], c1 = counts[p + 8], c2 = counts[p + 16], c3 = counts[p + 24];
    const float v0 = __ldg(partials + (size_t)p * kWgPart + off);
    const float v1 = __ldg(partials + (size_t)(p + 8) * kWgPart + off);
    const float v2 = __ldg(partials + (size_t)(p + 16) * kWgPart + off);
    const float v3 = __ldg(partials + (size_t)(p + 24) * kWgPart + off);
    if (c0) s += v0;
    if (c1) s += v1;
    if (c2) s += v2;
    if (c3) s += v3;
  }
  for (; p < nparts; p += 8)
    if (counts[p]) s += __ldg(partials + (size_t)p * kWgPart + off);
  red[g][l] = s;
  __syncthreads();
  if (g == 0)
    dW[((co * kC + ci) * 3 + kh) * 3 + kw] =
        ((red[0][l] + red[1][l]) + (red[2][l] + red[3][l])) + ((red[4][l] + red[5][l]) + (red[6][l] + red[7][l]));
}

int conv_wgrad_tc(const float* X, const float* dY, float* dW, const ConvShape& s, cudaStream_t st, bool* handled) {
  *handled = s.C == kC && s.K == kC && s.KH == 3 && s.KW == 3 && s.SH == 1 && s.SW == 1 && s.PH == 1 && s.PW == 1 &&
             s.W % 4 == 0 && (s.H * s.W) % 32 == 0 && s.N >= 1 && (long long)s.N * kC < (1 << 30) &&
             !(((uintptr_t)X | (uintptr_t)dY) & 15);
  if (!*handled) return AMC_OK;
  const int nsm = num_sms();
  const size_t part_bytes = (size_t)nsm * kWgPart * sizeof(float);
  void* scratch = nullptr;
  int rc = conv_scratch(part_bytes + 4096, &scratch);
  if (rc) return rc;
  float* parts = (float*)scratch;
  int* counts = (int*)(parts + (size_t)nsm * kWgPart);
  const int HW = s.H * s.W, cpi = HW / 32, total = s.N * cpi;
  const int grid = total < nsm ? total : nsm;
  std::vector<int> cnt(grid);
  for (int b = 0; b < grid; ++b)
    cnt[b] = (int)((long long)total * (b + 1) / grid) - (int)((long long)total * b / grid);
  AMC_CUDA(cudaMemcpyAsync(counts, cnt.data(), grid * sizeof(int), cudaMemcpyHostToDevice, st));
  CUtensorMap mDY, mX, mXh;
  const uint64_t rows = (uint64_t)s.N * kC;
  rc = make_tmap_2d_f32(&mDY, dY, rows, (uint64_t)HW, (uint64_t)HW, 64);
  if (!rc) rc = make_tmap_2d_f32(&mX, X, rows, (uint64_t)HW, (uint64_t)HW, 64);
  if (!rc) rc = make_tmap_2d_f32_box(&mXh, X, rows, (uint64_t)HW, (uint64_t)HW, 4, 64, false);
  if (rc) return rc;
  static std::atomic<uint64_t> attr{0};
  rc = smem_attr_once(k_conv_wgrad_tc, kWgSmem, attr);
  if (rc) return rc;
  k_conv_wgrad_tc<<<grid, 256, kWgSmem, st>>>(mDY, mX, mXh, parts, s.N, HW, s.W, cpi);
  AMC_CUDA(cudaGetLastError());
  k_wgrad_reduce<<<kC * kC * 9 / 32, 256, 0, st>>>(parts, dW, grid, counts);
  AMC_CUDA(cudaGetLastError());
  return AMC_OK;
}

int conv_check_error() {
  int e = 0;
  AMC_CUDA(cudaMemcpyFromSymbol(&e, g_conv_error, sizeof(int)));
  if (e) {
    int z = 0;
    AMC_CUDA(cudaMemcpyToSymbol(g_conv_error, &z, sizeof(int)));
    return fail(e, "conv: a bounded wait on the tensor-core pipeline gave up");
  }
  return AMC_OK;
}

}  // namespace amc
