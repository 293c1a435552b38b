// Linear-regression training step (f64): the replayed SSA program of
//   loss = mean((X w - y)^2),  dw = X^T dr,  dr = g*r + g*r,  g = 1/N
// (ssa.scm:517-1033 matmul/mean/mul rules; replay ssa.scm:1519-1654) fused
// into ONE pass over X per step.  The reference realizes the forward GEMV, the
// residual, the square, the mean, the broadcast gradient and the transposed
// GEMM as separate materialised nodes, reading X twice; here each warp reads a
// row of X once, forms its residual from a warp-wide dot product and folds the
// row into the gradient accumulators it already holds in registers.
#include "amc_internal.h"

namespace amc {

constexpr int kLinregBlock = 256;

static int linreg_grid(int64_t rows) {
  long long g = (long long)num_sms() * 4;
  long long need = (rows + 31) / 32;  // at least 32 rows per block
  if (need < g) g = need;
  return (int)(g < 1 ? 1 : g);
}

// KPL = columns per lane (d = 32 * KPL).
template <int KPL>
__global__ void __launch_bounds__(kLinregBlock) k_linreg_partials(const double* __restrict__ X, const double* __restrict__ y,
                                                                  const double* __restrict__ w, long long rows, double g,
                                                                  double* __restrict__ partials) {
  constexpr int D = 32 * KPL;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = kLinregBlock / 32;
  const long long gw = (long long)blockIdx.x * nw + warp, tw = (long long)gridDim.x * nw;
  const long long r0 = rows * gw / tw, r1 = rows * (gw + 1) / tw;
  double wv[KPL], acc[KPL];
#pragma unroll
  for (int j = 0; j < KPL; ++j) { wv[j] = __ldg(w + lane + 32 * j); acc[j] = 0.0; }
  double loss = 0.0;
  long long i = r0;
  // two rows per iteration: loads of the second row overlap the reduction of the first
  for (; i + 1 < r1; i += 2) {
    double xa[KPL], xb[KPL];
    const double* pa = X + i * D + lane;
#pragma unroll
    for (int j = 0; j < KPL; ++j) { xa[j] = __ldcs(pa + 32 * j); xb[j] = __ldcs(pa + D + 32 * j); }
    double ya = __ldg(y + i), yb = __ldg(y + i + 1);
    double pa_ = 0.0, pb_ = 0.0;
#pragma unroll
    for (int j = 0; j < KPL; ++j) { pa_ = fma(xa[j], wv[j], pa_); pb_ = fma(xb[j], wv[j], pb_); }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      pa_ += __shfl_xor_sync(0xffffffffu, pa_, o);
      pb_ += __shfl_xor_sync(0xffffffffu, pb_, o);
    }
    double ra = pa_ - ya, rb = pb_ - yb;
    double ga = g * ra, gb = g * rb;
    double da = ga + ga, db = gb + gb;
#pragma unroll
    for (int j = 0; j < KPL; ++j) acc[j] = fma(xb[j], db, fma(xa[j], da, acc[j]));
    loss = fma(rb, rb, fma(ra, ra, loss));
  }
  for (; i < r1; ++i) {
    double xa[KPL];
    const double* pa = X + i * D + lane;
#pragma unroll
    for (int j = 0; j < KPL; ++j) xa[j] = __ldcs(pa + 32 * j);
    double p = 0.0;
#pragma unroll
    for (int j = 0; j < KPL; ++j) p = fma(xa[j], wv[j], p);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) p += __shfl_xor_sync(0xffffffffu, p, o);
    double r = p - __ldg(y + i), gr = g * r, dr = gr + gr;
#pragma unroll
    for (int j = 0; j < KPL; ++j) acc[j] = fma(xa[j], dr, acc[j]);
    loss = fma(r, r, loss);
  }
  // block combine in warp order (fixed)
  __shared__ double sm[kLinregBlock / 32][D + 1];
#pragma unroll
  for (int j = 0; j < KPL; ++j) sm[warp][lane + 32 * j] = acc[j];
  if (lane == 0) sm[warp][D] = loss;
  __syncthreads();
  for (int k = threadIdx.x; k <= D; k += kLinregBlock) {
    double s = 0.0;
    for (int ww = 0; ww < nw; ++ww) s += sm[ww][k];
    partials[(long long)blockIdx.x * (D + 1) + k] = s;
  }
}

// Generic column count (d <= 1024): lanes stride over columns.
__global__ void __launch_bounds__(kLinregBlock) k_linreg_partials_any(const double* __restrict__ X, const double* __restrict__ y,
                                                                      const double* __restrict__ w, long long rows, int d,
                                                                      double g, double* __restrict__ partials) {
  extern __shared__ double smd[];  // [nw][d+1]
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = kLinregBlock / 32;
  const long long gw = (long long)blockIdx.x * nw + warp, tw = (long long)gridDim.x * nw;
  const long long r0 = rows * gw / tw, r1 = rows * (gw + 1) / tw;
  double* acc = smd + (size_t)warp * (d + 1);
  for (int k = lane; k <= d; k += 32) acc[k] = 0.0;
  __syncwarp();
  double loss = 0.0;
  for (long long i = r0; i < r1; ++i) {
    double p = 0.0;
    for (int k = lane; k < d; k += 32) p = fma(X[i * d + k], w[k], p);
    for (int o = 16; o > 0; o >>= 1) p += __shfl_xor_sync(0xffffffffu, p, o);
    double r = p - y[i], gr = g * r, dr = gr + gr;
    for (int k = lane; k < d; k += 32) acc[k] = fma(X[i * d + k], dr, acc[k]);
    loss = fma(r, r, loss);
  }
  if (lane == 0) acc[d] = loss;
  __syncthreads();
  for (int k = threadIdx.x; k <= d; k += kLinregBlock) {
    double s = 0.0;
    for (int ww = 0; ww < nw; ++ww) s += smd[(size_t)ww * (d + 1) + k];
    partials[(long long)blockIdx.x * (d + 1) + k] = s;
  }
}

// Sum of the n partial rows in a fixed order: a block takes 32 columns and 8
// groups of rows; group g adds rows g, g+8, ... in ascending order, then the
// 8 group sums are added in index order.  The loads of a group are
// independent of the other groups', so the sum is not one n-long dependent
// chain of loads.
__global__ void __launch_bounds__(256) k_linreg_reduce(const double* __restrict__ partials, int n, int d,
                                                       double* __restrict__ out) {
  __shared__ double red[8][33];
  const int l = threadIdx.x & 31, g = threadIdx.x >> 5;
  const int k = blockIdx.x * 32 + l;
  double s = 0.0;
  if (k <= d)
    for (int b = g; b < n; b += 8) s += __ldg(partials + (long long)b * (d + 1) + k);
  red[g][l] = s;
  __syncthreads();
  if (g == 0 && k <= d)
    out[k] = ((red[0][l] + red[1][l]) + (red[2][l] + red[3][l])) + ((red[4][l] + red[5][l]) + (red[6][l] + red[7][l]));
}

__global__ void k_linreg_update(double* __restrict__ w, const double* __restrict__ gl, int d, double n_total, double lr,
                                double* __restrict__ loss_out) {
  int k = blockIdx.x * blockDim.x + threadIdx.x;
  if (k < d) w[k] = w[k] - lr * gl[k];
  if (k == 0 && loss_out) *loss_out = gl[d] / n_total;
}

}  // namespace amc

using namespace amc;

extern "C" {

int amc_linreg_partials_count(int64_t rows, int32_t d, int32_t* n) {
  if (!n || rows < 0 || d <= 0) return fail(AMC_ERR_INVALID, "amc_linreg_partials_count: bad arguments");
  *n = linreg_grid(rows);
  return AMC_OK;
}

int amc_linreg_partials(const double* X, const double* y, const double* w, int64_t rows, int32_t d, int64_t n_total,
                        double* partials, void* stream) {
  if (!X || !y || !w || !partials || rows < 0 || d <= 0 || d > 1024 || n_total <= 0)
    return fail(AMC_ERR_INVALID, "amc_linreg_partials: bad arguments");
  if (fault_injected("launch")) return fail(AMC_ERR_INJECTED, "linreg: injected launch failure (AMC_FAULT=launch)");
  cudaStream_t s = pick_stream(stream);
  int grid = linreg_grid(rows);
  double g = 1.0 / (double)n_total;
  switch (d) {
    case 32: k_linreg_partials<1><<<grid, kLinregBlock, 0, s>>>(X, y, w, rows, g, partials); break;
    case 64: k_linreg_partials<2><<<grid, kLinregBlock, 0, s>>>(X, y, w, rows, g, partials); break;
    case 128: k_linreg_partials<4><<<grid, kLinregBlock, 0, s>>>(X, y, w, rows, g, partials); break;
    case 256: k_linreg_partials<8><<<grid, kLinregBlock, 0, s>>>(X, y, w, rows, g, partials); break;
    default: {
      size_t sm = (size_t)(kLinregBlock / 32) * (d + 1) * sizeof(double);
      if (sm > 48 * 1024) AMC_CUDA(cudaFuncSetAttribute(k_linreg_partials_any, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm));
      k_linreg_partials_any<<<grid, kLinregBlock, sm, s>>>(X, y, w, rows, d, g, partials);
    }
  }
  AMC_CUDA(cudaGetLastError());
  return AMC_OK;
}

int amc_linreg_reduce(const double* partials, int32_t n, int32_t d, double* grad_loss, void* stream) {
  if (!partials || !grad_loss || n <= 0 || d <= 0) return fail(AMC_ERR_INVALID, "amc_linreg_reduce: bad arguments");
  k_linreg_reduce<<<(d + 1 + 31) / 32, 256, 0, pick_stream(stream)>>>(partials, n, d, grad_loss);
  AMC_CUDA(cudaGetLastError());
  return AMC_OK;
}

int amc_linreg_update(double* w, const double* gl, int32_t d, int64_t n_total, double lr, double* loss_out, void* stream) {
  if (!w || !gl || d <= 0 || n_total <= 0) return fail(AMC_ERR_INVALID, "amc_linreg_update: bad arguments");
  k_linreg_update<<<(d + 127) / 128, 128, 0, pick_stream(stream)>>>(w, gl, d, (double)n_total, lr, loss_out);
  AMC_CUDA(cudaGetLastError());
  return AMC_OK;
}

int amc_linreg_step(const double* X, const double* y, double* w, int64_t rows, int32_t d, double lr, double* partials,
                    double* grad_loss, double* loss_out, void* stream) {
  int32_t n = 0;
  int rc = amc_linreg_partials_count(rows, d, &n);
  if (rc) return rc;
  rc = amc_linreg_partials(X, y, w, rows, d, rows, partials, stream);
  if (rc) return rc;
  rc = amc_linreg_reduce(partials, n, d, grad_loss, stream);
  if (rc) return rc;
  return amc_linreg_update(w, grad_loss, d, rows, lr, loss_out, stream);
}

}  // extern "C"
