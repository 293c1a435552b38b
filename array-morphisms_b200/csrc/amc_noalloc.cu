// Linear-regression step for callers that cannot allocate device memory.
//
// amc_linreg_step needs caller-provided scratch (per-block partial sums and
// the reduced gradient).  Some hosts cannot provide it: their device memory
// is owned by another allocator (a framework's caching allocator, a fixed
// per-process budget), or they must not call cudaMalloc inside a timed loop,
// where it can synchronise the device.  This variant keeps its scratch in a
// file-scope __device__ array of fixed size, loaded with the library on
// every GPU that loads it, and allocates nothing: no cudaMalloc, cudaFree or
// allocating library routine.
#include "amc_internal.h"

namespace amc {

// 2 MiB: partials (one row of d+1 doubles per block of the partials launch)
// plus the reduced gradient-and-loss row.
constexpr int64_t kNoallocScratchDoubles = 262144;

static __device__ __align__(256) double g_linreg_scratch[kNoallocScratchDoubles];

static std::mutex g_scratch_mu;
static std::unordered_map<int, double*> g_scratch_addr;

// The array's name in host code is a host-side stand-in, not a device
// address; the device address is looked up once per device, with that device
// current, and cached.
static int scratch_for_current_device(double** out) {
  int dev = 0;
  AMC_CUDA(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> l(g_scratch_mu);
  auto it = g_scratch_addr.find(dev);
  if (it != g_scratch_addr.end()) {
    *out = it->second;
    return AMC_OK;
  }
  double* p = nullptr;
  cudaError_t e = cudaGetSymbolAddress((void**)&p, g_linreg_scratch);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(linreg scratch)");
  g_scratch_addr[dev] = p;
  *out = p;
  return AMC_OK;
}

}  // namespace amc

using namespace amc;

extern "C" int amc_linreg_step_noalloc(const double* X, const double* y, double* w, int64_t rows, int32_t d, double lr,
                                       double* loss_out, void* stream) {
  if (!X || !y || !w || rows <= 0 || d <= 0) return fail(AMC_ERR_INVALID, "amc_linreg_step_noalloc: bad arguments");
  int32_t n = 0;
  int rc = amc_linreg_partials_count(rows, d, &n);
  if (rc) return rc;
  const int64_t need = ((int64_t)n + 1) * (int64_t)(d + 1);
  if (need > kNoallocScratchDoubles)
    return fail(AMC_ERR_INVALID, "amc_linreg_step_noalloc: needs " + std::to_string(need) +
                                     " scratch doubles ((partials + 1) * (d + 1)); the static scratch holds " +
                                     std::to_string(kNoallocScratchDoubles) + " (use amc_linreg_step with your own scratch)");
  double* scratch = nullptr;
  rc = scratch_for_current_device(&scratch);
  if (rc) return rc;
  double* partials = scratch;                            // n * (d + 1), every entry written by the partials launch
  double* grad_loss = scratch + (int64_t)n * (d + 1);    // d + 1, every entry written by the reduce launch
  rc = amc_linreg_partials(X, y, w, rows, d, rows, partials, stream);
  if (rc) return rc;
  rc = amc_linreg_reduce(partials, n, d, grad_loss, stream);
  if (rc) return rc;
  return amc_linreg_update(w, grad_loss, d, rows, lr, loss_out, stream);
}
