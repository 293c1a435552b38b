// Tensor-core throughput probe: the TF32 roofline denominator measured on
// the running GPU, and the issue-rate table behind the kernels' tile shapes.
// One CTA per SM; `warps` threads (lane 0 of warps 0..warps-1) each issue
// back-to-back tcgen05.mma kind::tf32 of M=128, N=n, K=8 into their own
// tensor-memory accumulator.  B is always in shared memory; A is in shared
// memory (a_tmem = 0) or in tensor memory (a_tmem = 1, the ts form).  The
// products' FLOPs over the event-timed duration give the rate.  With n=256
// one issuing thread is faster than the pipe, so that figure is the dense
// TF32 peak; smaller n show what bounds narrow products (shared-memory
// operand bytes per product against the pipe).  Diagnostic only: no
// reference counterpart.
#include "amc_internal.h"
#include "amc_tc.cuh"

namespace amc {

using namespace tc;

namespace {
// A 128 rows and B 256 rows of 128 B, barriers, alignment; sized above half
// the SM's shared memory so exactly one CTA runs per SM
constexpr int kPeakSmem = 120 * 1024;
__device__ int g_peak_error;
__device__ int g_wait_probe_error;
}  // namespace

// The bounded mbarrier wait every TMA/tensor-core kernel uses, on its own:
// one thread initialises a barrier that expects one arrival, arrives on it
// only when `arrive` is set, and waits with the given poll limit.  With no
// arrival the wait runs out, the thread records AMC_ERR_TIMEOUT in the flag
// and the kernel returns, as the production kernels do on expiry.
__global__ void k_wait_probe(int limit, int arrive) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x != 0) return;
  mbar_init(&bar, 1);
  mbar_fence_init();
  if (arrive) mbar_arrive(&bar);
  if (!mbar_wait(&bar, 0, limit)) atomicExch(&g_wait_probe_error, AMC_ERR_TIMEOUT);
}

template <int N, bool ATMEM>
__global__ void __launch_bounds__(128, 1) k_tc_peak(int iters, int warps) {
  extern __shared__ unsigned char peak_sm_raw[];
  unsigned char* sm = (unsigned char*)(((uintptr_t)peak_sm_raw + 1023) & ~(uintptr_t)1023);
  uint64_t* bar = (uint64_t*)(sm + 49152);   // [4]
  uint32_t* slot = (uint32_t*)(sm + 49152 + 64);
  const int tid = threadIdx.x, warp = tid >> 5;
  for (int i = tid; i < 49152 / 4; i += 128) reinterpret_cast<float*>(sm)[i] = 0.0078125f * (float)(i & 7);
  if (tid == 0) {
    for (int i = 0; i < 4; ++i) mbar_init(&bar[i], 1);
    mbar_fence_init();
  }
  fence_proxy_async();
  __syncthreads();
  if (warp == 0) tmem_alloc(slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *slot;
  // ts form: A is 128 lanes x 32 columns at column 480 (4 K steps of 8)
  constexpr uint32_t kACol = 480;
  if (ATMEM) {
    float v[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = 0.0078125f * (float)(i & 7);
    tmem_st32(tmem + ((uint32_t)(warp * 32) << 16) + kACol, v);
    tmem_st_wait();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
  }
  if ((tid & 31) == 0 && warp < warps) {
    const uint32_t id = idesc_tf32(128, N, false, false);
    const uint64_t a0 = sdesc(smem_addr(sm), 16, 1024), b0 = sdesc(smem_addr(sm + 16384), 16, 1024);
    const uint32_t d = tmem + (uint32_t)(warp * N);
    if (ATMEM) {
      mma_tf32_ts(d, tmem + kACol, b0, id, false);
      for (int it = 0; it < iters; ++it) {
#pragma unroll
        for (int k = 0; k < 4; ++k) mma_tf32_ts(d, tmem + kACol + 8 * k, desc_add(b0, k * 32), id, true);
      }
    } else {
      mma_tf32(d, a0, b0, id, false);
      for (int it = 0; it < iters; ++it) {
#pragma unroll
        for (int k = 0; k < 4; ++k) mma_tf32(d, desc_add(a0, k * 32), desc_add(b0, k * 32), id, true);
      }
    }
    mma_commit(&bar[warp]);
    if (!mbar_wait(&bar[warp], 0, 1 << 26)) atomicExch(&g_peak_error, AMC_ERR_TIMEOUT);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, 512);
}

template <int N, bool ATMEM>
static int run_peak(int iters, int warps, cudaStream_t s, float* ms) {
  static std::atomic<uint64_t> attr{0};
  const int rc = smem_attr_once(k_tc_peak<N, ATMEM>, kPeakSmem, attr);
  if (rc) return rc;
  const int sms = num_sms();
  cudaEvent_t a, b;
  AMC_CUDA(cudaEventCreate(&a));
  AMC_CUDA(cudaEventCreate(&b));
  k_tc_peak<N, ATMEM><<<sms, 128, kPeakSmem, s>>>(iters / 4 + 1, warps);   // warm-up
  AMC_CUDA(cudaEventRecord(a, s));
  k_tc_peak<N, ATMEM><<<sms, 128, kPeakSmem, s>>>(iters, warps);
  AMC_CUDA(cudaEventRecord(b, s));
  cudaError_t e = cudaEventSynchronize(b);
  if (e == cudaSuccess) e = cudaEventElapsedTime(ms, a, b);
  cudaEventDestroy(a);
  cudaEventDestroy(b);
  if (e != cudaSuccess) return cuda_fail(e, "k_tc_peak");
  return AMC_OK;
}

}  // namespace amc

using namespace amc;

template <bool ATMEM>
static int run_peak_n(int n, int iters, int warps, cudaStream_t s, float* ms) {
  return n == 32 ? run_peak<32, ATMEM>(iters, warps, s, ms)
         : n == 64 ? run_peak<64, ATMEM>(iters, warps, s, ms)
         : n == 128 ? run_peak<128, ATMEM>(iters, warps, s, ms)
                    : run_peak<256, ATMEM>(iters, warps, s, ms);
}

extern "C" int amc_tc_peak_tf32(int32_t n, int32_t warps, int32_t a_tmem, int32_t iters, double* tflops, void* stream) {
  if (!tflops || iters <= 0 || iters > (1 << 20) || warps < 1 || warps > 4 || (a_tmem != 0 && a_tmem != 1) ||
      (n != 32 && n != 64 && n != 128 && n != 256) || n * warps > (a_tmem ? 480 : 512))
    return fail(AMC_ERR_INVALID,
                "amc_tc_peak_tf32: n in {32,64,128,256}, warps 1..4, a_tmem 0|1, n*warps <= 512 (480 with a_tmem)");
  cudaStream_t s = pick_stream(stream);
  float ms = 0.f;
  int rc = a_tmem ? run_peak_n<true>(n, iters, warps, s, &ms) : run_peak_n<false>(n, iters, warps, s, &ms);
  if (rc) return rc;
  int err = 0;
  AMC_CUDA(cudaMemcpyFromSymbol(&err, g_peak_error, sizeof(int)));
  if (err) {
    int z = 0;
    AMC_CUDA(cudaMemcpyToSymbol(g_peak_error, &z, sizeof(int)));
    return fail(err, "amc_tc_peak_tf32: the completion wait gave up");
  }
  const double flops = 2.0 * 128.0 * n * 8.0 * (4.0 * iters + 1.0) * warps * num_sms();
  *tflops = ms > 0.f ? flops / (ms * 1e-3) / 1e12 : 0.0;
  return AMC_OK;
}

extern "C" int amc_probe_bounded_wait(int32_t limit, int32_t arrive, void* stream) {
  if (limit < 1 || limit > (1 << 22) || (arrive != 0 && arrive != 1))
    return fail(AMC_ERR_INVALID, "amc_probe_bounded_wait: limit 1..2^22, arrive 0|1");
  cudaStream_t s = pick_stream(stream);
  k_wait_probe<<<1, 32, 0, s>>>(limit, arrive);
  AMC_CUDA(cudaGetLastError());
  AMC_CUDA(cudaStreamSynchronize(s));
  int err = 0;
  AMC_CUDA(cudaMemcpyFromSymbol(&err, g_wait_probe_error, sizeof(int)));
  if (err) {
    int z = 0;
    AMC_CUDA(cudaMemcpyToSymbol(g_wait_probe_error, &z, sizeof(int)));
    return fail(err, "amc_probe_bounded_wait: the wait gave up after " + std::to_string(limit) + " polls");
  }
  return AMC_OK;
}
