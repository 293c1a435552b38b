// Tensor-core throughput probe: the TF32 roofline denominator measured on
// the running GPU.  One CTA per SM issues back-to-back tcgen05.mma
// kind::tf32 of M=128, N=256, K=8 (operands resident in shared memory, the
// accumulator in tensor memory) from one thread; the products' FLOPs over
// the event-timed duration give the reachable dense TF32 rate.  N=256 is the
// shape whose issue cost is below its tensor-pipe time, so the figure is the
// pipe's, not the issuing thread's.  Diagnostic only: no reference
// counterpart.
#include "amc_internal.h"
#include "amc_tc.cuh"

namespace amc {

using namespace tc;

namespace {
constexpr int kPeakN = 256;
constexpr int kPeakSmem = 16384 + 32768 + 1024 + 1024;   // A 128 rows, B 256 rows (128 B each), barrier, alignment
__device__ int g_peak_error;
}  // namespace

__global__ void __launch_bounds__(128, 1) k_tc_peak(int iters) {
  extern __shared__ unsigned char peak_sm_raw[];
  unsigned char* sm = (unsigned char*)(((uintptr_t)peak_sm_raw + 1023) & ~(uintptr_t)1023);
  uint64_t* bar = (uint64_t*)(sm + 49152);
  uint32_t* slot = (uint32_t*)(sm + 49152 + 64);
  const int tid = threadIdx.x;
  for (int i = tid; i < 49152 / 4; i += 128) reinterpret_cast<float*>(sm)[i] = 0.0078125f * (float)(i & 7);
  if (tid == 0) {
    mbar_init(bar, 1);
    mbar_fence_init();
  }
  fence_proxy_async();
  __syncthreads();
  if (tid < 32) tmem_alloc(slot, kPeakN);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *slot;
  if (tid == 0) {
    const uint32_t id = idesc_tf32(128, kPeakN, false, false);
    const uint64_t a0 = sdesc(smem_addr(sm), 16, 1024), b0 = sdesc(smem_addr(sm + 16384), 16, 1024);
    mma_tf32(tmem, a0, b0, id, false);
    for (int it = 0; it < iters; ++it) {
#pragma unroll
      for (int k = 0; k < 4; ++k) mma_tf32(tmem, desc_add(a0, k * 32), desc_add(b0, k * 32), id, true);
    }
    mma_commit(bar);
    if (!mbar_wait(bar, 0, 1 << 26)) atomicExch(&g_peak_error, AMC_ERR_TIMEOUT);
  }
  tc_fence_before();
  __syncthreads();
  if (tid < 32) tmem_dealloc(tmem, kPeakN);
}

}  // namespace amc

using namespace amc;

extern "C" int amc_tc_peak_tf32(int32_t iters, double* tflops, void* stream) {
  if (!tflops || iters <= 0 || iters > (1 << 20)) return fail(AMC_ERR_INVALID, "amc_tc_peak_tf32: bad arguments");
  cudaStream_t s = pick_stream(stream);
  static bool attr = false;
  if (!attr) {
    AMC_CUDA(cudaFuncSetAttribute(k_tc_peak, cudaFuncAttributeMaxDynamicSharedMemorySize, kPeakSmem));
    attr = true;
  }
  const int sms = num_sms();
  cudaEvent_t a, b;
  AMC_CUDA(cudaEventCreate(&a));
  AMC_CUDA(cudaEventCreate(&b));
  k_tc_peak<<<sms, 128, kPeakSmem, s>>>(iters / 4 + 1);   // warm-up
  AMC_CUDA(cudaEventRecord(a, s));
  k_tc_peak<<<sms, 128, kPeakSmem, s>>>(iters);
  AMC_CUDA(cudaEventRecord(b, s));
  cudaError_t e = cudaEventSynchronize(b);
  float ms = 0.f;
  if (e == cudaSuccess) e = cudaEventElapsedTime(&ms, a, b);
  cudaEventDestroy(a);
  cudaEventDestroy(b);
  if (e != cudaSuccess) return cuda_fail(e, "k_tc_peak");
  int err = 0;
  AMC_CUDA(cudaMemcpyFromSymbol(&err, g_peak_error, sizeof(int)));
  if (err) {
    int z = 0;
    AMC_CUDA(cudaMemcpyToSymbol(g_peak_error, &z, sizeof(int)));
    return fail(err, "amc_tc_peak_tf32: the completion wait gave up");
  }
  const double flops = 2.0 * 128.0 * kPeakN * 8.0 * (4.0 * iters + 1.0) * sms;
  *tflops = ms > 0.f ? flops / (ms * 1e-3) / 1e12 : 0.0;
  return AMC_OK;
}
