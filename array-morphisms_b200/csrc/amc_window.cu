// Windowed FIR reduction: the polyphase filter-bank tree
//   morph-reduce 'sum (morph* (transpose (reshape (im2col x (1 KW) (1 S)))) h) over taps
// lowered to one kernel.  With hop S equal to the branch count M the window of
// frame f+1 is the window of frame f shifted by one M-wide row, so
//   out[b, f, m] = sum_{t<16} h[t, m] * x[b, (f + t) * M + m]
// is a 16-tap FIR along the row axis of the (rows, M) matrix view of x.
//
// Each warp streams the rows of one chunk of frames once.  Row j contributes
// tap t to frame j - t; the 16 frames in flight live in a register ring,
// indexed statically by unrolling 16 rows at a time, and frame j - 15 is
// complete (all taps added, in ascending t) after row j.  Each lane owns two
// branches (8-byte loads and stores); arithmetic keeps separate multiply and
// add roundings: acc = fl(acc + fl(h * x)) from +0.0, which is bit-identical to
// the reference's per-node materialisation (f32 product node, then f32
// partial sums re-read from the typed output, realization.scm:1309-1388).
#include "amc_internal.h"

namespace amc {

constexpr int kTaps = 16;
constexpr int kChunk = 256;  // frames per warp (multiple of 16)

__device__ __forceinline__ float2 ldg2(const float2* p) { return __ldg(p); }

// One tap of two branches: acc = fl(acc + fl(h * x)) per component.  Scalar
// mul.rn / add.rn are never contracted; the packed f32x2 forms (intrinsics or
// explicit .rn PTX) were measured to come out fused on this toolchain, which
// changes the rounding, so they are not used here.
__device__ __forceinline__ float2 tap2(float2 acc, float2 h, float2 x) {
  return make_float2(__fadd_rn(acc.x, __fmul_rn(h.x, x.x)), __fadd_rn(acc.y, __fmul_rn(h.y, x.y)));
}
// First tap of a frame: the reference's output starts at +0.0, so the first
// partial is fl(+0.0 + fl(h * x)) (which turns a -0.0 product into +0.0).
__device__ __forceinline__ float2 tap2_first(float2 h, float2 x) {
  return make_float2(__fadd_rn(0.f, __fmul_rn(h.x, x.x)), __fadd_rn(0.f, __fmul_rn(h.y, x.y)));
}

template <int PHASE>  // 0: rows 0..15 of the chunk; 1: interior; 2: rows chunk..chunk+14
__device__ __forceinline__ void fir_rows16(float2 (&acc)[kTaps], const float2 (&h)[kTaps],
                                           const float2* __restrict__ xrow, long long xs,
                                           float2* __restrict__ orow, long long os, bool store_ok) {
  float2 xv[16];
#pragma unroll
  for (int jj = 0; jj < 16; ++jj) {
    if (PHASE == 2 && jj == 15) continue;
    xv[jj] = ldg2(xrow + jj * xs);
  }
#pragma unroll
  for (int jj = 0; jj < 16; ++jj) {
    if (PHASE == 2 && jj == 15) continue;
#pragma unroll
    for (int t = 0; t < kTaps; ++t) {
      const bool valid = PHASE == 0 ? (t <= jj) : PHASE == 2 ? (t > jj) : true;
      if (valid) {
        const int slot = (jj - t) & 15;
        acc[slot] = tap2(acc[slot], h[t], xv[jj]);
      }
    }
    const bool done = PHASE == 0 ? (jj == 15) : true;
    if (done) {
      const int slot = (jj + 1) & 15;
      // frame (row - 15): orow points at the frame of row index 0 of this group minus 15
      if (store_ok) __stcs(orow + jj * os, acc[slot]);
      acc[slot] = make_float2(0.f, 0.f);
    }
  }
}

// ------------------------------------------------------------------ TMA-staged variant
// Rows are contiguous when hop == branches, so the rows of a chunk form one
// contiguous span of global memory.  Each warp keeps a ring of kStages tiles
// of 16 rows in shared memory; lane 0 fills them with 1-D bulk async copies
// (cp.async.bulk, completion counted on an mbarrier per stage, no multicast)
// kStages groups ahead of the arithmetic, so the memory pipeline never waits
// for registers.  Every mbarrier wait is bounded: on expiry the kernel records
// an error code, drains its own copies (also bounded) and returns.
constexpr int kStages = 4;
constexpr int kWarpsPerCta = 4;
constexpr int kWaitLimit = 1 << 20;

static __device__ int g_fir_error;

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t phase) {
  for (int i = 0; i < kWaitLimit; ++i) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok) : "r"(bar), "r"(phase) : "memory");
    if (ok) return true;
  }
  return false;
}

__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               ::"r"(dst), "l"(src), "r"(bytes), "r"(bar) : "memory");
}

// RS: row stride of the staged tile and frame stride of the output, in float2
// (compile-time for the 64-branch bank so every access uses an immediate offset).
template <int PHASE, int RS>
__device__ __forceinline__ void fir_rows16_smem(float2 (&acc)[kTaps], const float2 (&h)[kTaps],
                                                const float2* __restrict__ srow, int rs_rt,
                                                float2* __restrict__ orow, long long os_rt, bool store_ok) {
  const int rs = RS ? RS : rs_rt;
  const long long os = RS ? RS : os_rt;
  float2 xv[16];
#pragma unroll
  for (int jj = 0; jj < 16; ++jj) {
    if (PHASE == 2 && jj == 15) continue;
    xv[jj] = srow[jj * rs];
  }
#pragma unroll
  for (int jj = 0; jj < 16; ++jj) {
    if (PHASE == 2 && jj == 15) continue;
#pragma unroll
    for (int t = 0; t < kTaps; ++t) {
      const bool valid = PHASE == 0 ? (t <= jj) : PHASE == 2 ? (t > jj) : true;
      if (valid) {
        const int slot = (jj - t) & 15;
        acc[slot] = t == 0 ? tap2_first(h[t], xv[jj]) : tap2(acc[slot], h[t], xv[jj]);
      }
    }
    const bool done = PHASE == 0 ? (jj == 15) : true;
    if (done && store_ok) __stcs(orow + jj * os, acc[(jj + 1) & 15]);
  }
}

template <int RS>
__global__ void __launch_bounds__(kWarpsPerCta * 32) k_fir_tma(const __grid_constant__ FirArgs a, long long chunks_per_sig) {
  extern __shared__ __align__(128) unsigned char fir_sm[];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const long long warp = (long long)blockIdx.x * kWarpsPerCta + w;
  const long long items = a.batch * chunks_per_sig;
  if (warp >= items) return;
  const int RB = a.branches * 4;          // bytes per row
  const int SB = 16 * RB;                 // bytes per stage
  const int rs = a.branches >> 1;         // row stride in float2
  unsigned char* ring = fir_sm + (size_t)w * kStages * SB;
  uint64_t* bars = reinterpret_cast<uint64_t*>(fir_sm + (size_t)kWarpsPerCta * kStages * SB) + w * kStages;
  const int pairs = a.branches >> 1;
  const bool active = lane < pairs;
  const int q = active ? lane : 0;
  const long long b = warp / chunks_per_sig, c = warp % chunks_per_sig;
  const long long f0 = c * kChunk;
  const char* src = reinterpret_cast<const char*>(a.x + b * a.x_bstride + f0 * a.hop);
  constexpr int kRows = kChunk + kTaps - 1;
  constexpr int kGroups = (kRows + 15) / 16;
  if (lane == 0) {
    for (int s = 0; s < kStages; ++s)
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(&bars[s])) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    for (int g = 0; g < kStages && g < kGroups; ++g) {
      const int rows = (g == kGroups - 1) ? kRows - 16 * g : 16;
      bulk_load(smem_u32(ring + (size_t)g * SB), src + (size_t)g * 16 * RB, (uint32_t)(rows * RB), smem_u32(&bars[g]));
    }
  }
  __syncwarp();
  const long long os = a.o_fstride >> 1;
  float2* obase = reinterpret_cast<float2*>(a.out + b * a.o_bstride + f0 * a.o_fstride) + q;
  float2 h[kTaps], acc[kTaps];
#pragma unroll
  for (int t = 0; t < kTaps; ++t) {
    h[t] = ldg2(reinterpret_cast<const float2*>(a.h + t * a.h_tstride) + q);
    acc[t] = make_float2(0.f, 0.f);
  }
#pragma unroll 1
  for (int g = 0; g < kGroups; ++g) {
    const int s = g % kStages;
    const uint32_t phase = (uint32_t)(g / kStages) & 1u;
    if (!mbar_wait(smem_u32(&bars[s]), phase)) {
      if (lane == 0) atomicExch(&g_fir_error, AMC_ERR_TIMEOUT);
      // drain this warp's other copies in flight (bounded), then leave
      for (int k = g + 1; k < g + kStages && k < kGroups; ++k)
        mbar_wait(smem_u32(&bars[k % kStages]), (uint32_t)(k / kStages) & 1u);
      return;
    }
    const float2* srow = reinterpret_cast<const float2*>(ring + (size_t)s * SB) + q;
    float2* orow = obase + ((long long)g * 16 - 15) * os;
    if (g == 0) fir_rows16_smem<0, RS>(acc, h, srow, rs, orow, os, active);
    else if (g < kGroups - 1) fir_rows16_smem<1, RS>(acc, h, srow, rs, orow, os, active);
    else fir_rows16_smem<2, RS>(acc, h, srow, rs, orow, os, active);
    __syncwarp();
    if (lane == 0 && g + kStages < kGroups) {
      const int gn = g + kStages;
      const int rows = (gn == kGroups - 1) ? kRows - 16 * gn : 16;
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      bulk_load(smem_u32(ring + (size_t)s * SB), src + (size_t)gn * 16 * RB, (uint32_t)(rows * RB), smem_u32(&bars[s]));
    }
  }
}

// One warp per (signal, chunk of kChunk frames); lane q owns branches 2q, 2q+1.
__global__ void __launch_bounds__(256, 2) k_fir_chunks(const __grid_constant__ FirArgs a, long long chunks_per_sig) {
  const int lane = threadIdx.x & 31;
  const long long warp = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const long long items = a.batch * chunks_per_sig;
  if (warp >= items) return;
  const int pairs = a.branches >> 1;
  const bool active = lane < pairs;
  const int q = active ? lane : 0;
  const long long b = warp / chunks_per_sig, c = warp % chunks_per_sig;
  const long long f0 = c * kChunk;
  const long long xs = a.hop >> 1, os = a.o_fstride >> 1;  // strides in float2 units
  const float2* xbase = reinterpret_cast<const float2*>(a.x + b * a.x_bstride + f0 * a.hop) + q;
  float2* obase = reinterpret_cast<float2*>(a.out + b * a.o_bstride + f0 * a.o_fstride) + q;
  float2 h[kTaps], acc[kTaps];
#pragma unroll
  for (int t = 0; t < kTaps; ++t) {
    h[t] = ldg2(reinterpret_cast<const float2*>(a.h + t * a.h_tstride) + q);
    acc[t] = make_float2(0.f, 0.f);
  }
  // group 0: rows 0..15, completes frame 0 at row 15
  fir_rows16<0>(acc, h, xbase, xs, obase - 15 * os, os, active);
#pragma unroll 1
  for (int g = 1; g < kChunk / 16; ++g)
    fir_rows16<1>(acc, h, xbase + (long long)g * 16 * xs, xs, obase + ((long long)g * 16 - 15) * os, os, active);
  fir_rows16<2>(acc, h, xbase + (long long)kChunk * xs, xs, obase + ((long long)kChunk - 15) * os, os, active);
}

// Frames past the last full chunk: one thread per (signal, frame, branch pair),
// taps added in ascending order.
__global__ void k_fir_tail(const __grid_constant__ FirArgs a, long long fstart) {
  const int pairs = a.branches >> 1;
  const long long nf = a.frames - fstart;
  const long long total = a.batch * nf * pairs;
  long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= total) return;
  const int q = (int)(i % pairs);
  const long long f = fstart + (i / pairs) % nf, b = i / (pairs * nf);
  const float2* xr = reinterpret_cast<const float2*>(a.x + b * a.x_bstride + f * a.hop) + q;
  float2 acc = make_float2(0.f, 0.f);
  for (int t = 0; t < a.taps; ++t) {
    float2 hv = ldg2(reinterpret_cast<const float2*>(a.h + t * a.h_tstride) + q);
    acc = tap2(acc, hv, ldg2(xr + (long long)t * (a.x_tstride >> 1)));
  }
  reinterpret_cast<float2*>(a.out + b * a.o_bstride + f * a.o_fstride)[q] = acc;
}

static bool aligned8(const void* p) { return ((uintptr_t)p & 7) == 0; }

bool fir_supported(const FirArgs& a) {
  return a.taps == kTaps && a.branches >= 2 && a.branches <= 64 && (a.branches % 2) == 0 && a.hop == a.x_tstride &&
         (a.hop % 2) == 0 && (a.x_bstride % 2) == 0 && (a.h_tstride % 2) == 0 && (a.o_fstride % 2) == 0 &&
         (a.o_bstride % 2) == 0 && aligned8(a.x) && aligned8(a.h) && aligned8(a.out) && a.hop >= a.branches;
}

int fir_launches(const FirArgs& a) {
  if (a.batch == 0 || a.frames == 0) return 0;
  return (a.frames / kChunk > 0 ? 1 : 0) + (a.frames % kChunk ? 1 : 0);
}

// The bulk-copy kernel needs contiguous rows (hop == branches), rows of a
// multiple of 16 bytes and 16-byte aligned chunk starts.
static bool fir_tma_ok(const FirArgs& a) {
  const uintptr_t x = (uintptr_t)a.x;
  return a.hop == a.branches && (a.branches * 4) % 16 == 0 && (x % 16) == 0 && ((a.x_bstride * 4) % 16) == 0 &&
         ((kChunk * a.hop * 4) % 16) == 0;
}

int fir_check_error() {
  int e = 0;
  AMC_CUDA(cudaMemcpyFromSymbol(&e, g_fir_error, sizeof(int)));
  if (e) {
    int z = 0;
    AMC_CUDA(cudaMemcpyToSymbol(g_fir_error, &z, sizeof(int)));
    return fail(e, "window FIR: a bounded wait for a staged tile gave up");
  }
  return AMC_OK;
}

int launch_fir(const FirArgs& a, cudaStream_t s) {
  if (!fir_supported(a)) return fail(AMC_ERR_UNSUPPORTED, "window FIR: layout not supported by the streaming kernel");
  if (fault_injected("launch")) return fail(AMC_ERR_INJECTED, "window FIR: injected launch failure (AMC_FAULT=launch)");
  if (a.batch == 0 || a.frames == 0) return AMC_OK;
  const long long chunks = a.frames / kChunk;
  if (chunks > 0) {
    const long long warps = a.batch * chunks;
    if (fir_tma_ok(a)) {
      const size_t sm = (size_t)kWarpsPerCta * kStages * 16 * a.branches * 4 + (size_t)kWarpsPerCta * kStages * 8;
      const unsigned blocks = (unsigned)((warps + kWarpsPerCta - 1) / kWarpsPerCta);
      if (a.branches == 64 && a.o_fstride == 64) {
        AMC_CUDA(cudaFuncSetAttribute(k_fir_tma<32>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm));
        k_fir_tma<32><<<blocks, kWarpsPerCta * 32, sm, s>>>(a, chunks);
      } else {
        AMC_CUDA(cudaFuncSetAttribute(k_fir_tma<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm));
        k_fir_tma<0><<<blocks, kWarpsPerCta * 32, sm, s>>>(a, chunks);
      }
    } else {
      const unsigned blocks = (unsigned)((warps + 7) / 8);
      k_fir_chunks<<<blocks, 256, 0, s>>>(a, chunks);
    }
    AMC_CUDA(cudaGetLastError());
  }
  const long long fstart = chunks * kChunk;
  if (fstart < a.frames) {
    const long long total = a.batch * (a.frames - fstart) * (a.branches / 2);
    k_fir_tail<<<(unsigned)((total + 255) / 256), 256, 0, s>>>(a, fstart);
    AMC_CUDA(cudaGetLastError());
  }
  return AMC_OK;
}

}  // namespace amc

using namespace amc;

extern "C" int amc_window_fir_f32(const float* x, int64_t batch, int64_t x_batch_stride, int64_t frames, int64_t hop,
                                  int32_t taps, int32_t branches, const float* h, float* out, void* stream) {
  if (!x || !h || !out || batch < 0 || frames < 0) return fail(AMC_ERR_INVALID, "amc_window_fir_f32: bad arguments");
  FirArgs a;
  a.x = x;
  a.batch = batch;
  a.x_bstride = x_batch_stride;
  a.frames = frames;
  a.hop = hop;
  a.taps = taps;
  a.branches = branches;
  a.x_tstride = branches;
  a.h = h;
  a.h_tstride = branches;
  a.out = out;
  a.o_fstride = branches;
  a.o_bstride = frames * branches;
  return launch_fir(a, pick_stream(stream));
}
