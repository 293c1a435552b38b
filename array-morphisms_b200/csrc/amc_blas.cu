// BLAS backend record entries (make-blas-backend slots, blas-exec.scm:16-46):
// the normalized kernel interface on host vectors, so a Scheme adapter can
// register libamcuda exactly as chicken-blas-backend.scm registers the CBLAS
// egg.  Operands are staged through stream-ordered device memory; the
// arithmetic is the planner's: the double-accumulating k_gemm, whose f64
// results match the reference's Scheme fallback loops bit for bit and whose
// f32 results are rounded once from double, and for large matrix-vector
// shapes and dot products the row passes of amc_rowpass.cu (double
// accumulation in a fixed parallel order).
#include <cstring>

#include "amc_internal.h"

namespace amc {

__global__ void k_axpy(long long n, double alpha, const void* x, void* y, int dtype) {
  long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  if (dtype == AMC_F64) {
    double* yy = (double*)y;
    yy[i] = __dadd_rn(__dmul_rn(alpha, ((const double*)x)[i]), yy[i]);
  } else {
    float* yy = (float*)y;
    yy[i] = __double2float_rn(__dadd_rn(__dmul_rn(alpha, (double)((const float*)x)[i]), (double)yy[i]));
  }
}

namespace {
struct Staging {
  cudaStream_t s;
  std::vector<void*> ptrs;
  int rc = AMC_OK;
  explicit Staging(cudaStream_t st) : s(st) {}
  void* up(const void* host, size_t bytes) {
    void* d = nullptr;
    if (rc) return nullptr;
    cudaError_t e = cudaMallocAsync(&d, bytes ? bytes : 16, s);
    if (e != cudaSuccess) { rc = cuda_fail(e, "cudaMallocAsync"); return nullptr; }
    ptrs.push_back(d);
    if (host && bytes) {
      e = cudaMemcpyAsync(d, host, bytes, cudaMemcpyHostToDevice, s);
      if (e != cudaSuccess) { rc = cuda_fail(e, "cudaMemcpyAsync"); return nullptr; }
    }
    return d;
  }
  int down(void* host, const void* d, size_t bytes) {
    if (rc) return rc;
    if (bytes) {
      cudaError_t e = cudaMemcpyAsync(host, d, bytes, cudaMemcpyDeviceToHost, s);
      if (e != cudaSuccess) rc = cuda_fail(e, "cudaMemcpyAsync");
    }
    return rc;
  }
  int finish() {
    for (void* p : ptrs) cudaFreeAsync(p, s);
    cudaError_t e = cudaStreamSynchronize(s);
    if (!rc && e != cudaSuccess) rc = cuda_fail(e, "cudaStreamSynchronize");
    return rc;
  }
};

int gemm_host(int dtype, int32_t M, int32_t N, int32_t K, double alpha, const void* A, int32_t lda, int32_t ta,
              const void* B, int32_t ldb, int32_t tb, double beta, void* C) {
  if (M < 0 || N < 0 || K < 0 || !A || !B || !C) return fail(AMC_ERR_INVALID, "gemm: bad arguments");
  if (fault_injected("launch")) return fail(AMC_ERR_INJECTED, "gemm: injected launch failure (AMC_FAULT=launch)");
  size_t es = dtype_size(dtype);
  Staging st(default_stream());
  size_t an = (size_t)(ta ? (int64_t)K * lda : (int64_t)M * lda), bn = (size_t)(tb ? (int64_t)N * ldb : (int64_t)K * ldb);
  if (M && K && an < (size_t)(ta ? (int64_t)(K - 1) * lda + M : (int64_t)(M - 1) * lda + K)) return fail(AMC_ERR_INVALID, "gemm: lda too small");
  if (K && N && bn < (size_t)(tb ? (int64_t)(N - 1) * ldb + K : (int64_t)(K - 1) * ldb + N)) return fail(AMC_ERR_INVALID, "gemm: ldb too small");
  // stage exactly the addressed span
  size_t a_span = (M && K) ? (size_t)(ta ? (int64_t)(K - 1) * lda + M : (int64_t)(M - 1) * lda + K) : 0;
  size_t b_span = (K && N) ? (size_t)(tb ? (int64_t)(N - 1) * ldb + K : (int64_t)(K - 1) * ldb + N) : 0;
  void* dA = st.up(A, a_span * es);
  void* dB = st.up(B, b_span * es);
  void* dC = st.up(beta != 0.0 ? C : nullptr, (size_t)M * N * es);
  if (st.rc) return st.finish();
  GemmArgs g;
  memset(&g, 0, sizeof g);
  g.M = M; g.N = N; g.K = K;
  g.A = dA; g.a_dtype = dtype; g.sa0 = ta ? 1 : lda; g.sa1 = ta ? lda : 1;
  g.B = dB; g.b_dtype = dtype; g.sb0 = tb ? 1 : ldb; g.sb1 = tb ? ldb : 1;
  g.C = dC; g.c_dtype = dtype;
  g.alpha = alpha; g.beta = beta;
  void* scratch = nullptr;
  if (size_t sb = gemm_scratch_bytes(g)) scratch = st.up(nullptr, sb);
  if (st.rc) return st.finish();
  int rc = launch_gemm_scratch(g, scratch, st.s);
  if (rc) { st.rc = rc; return st.finish(); }
  st.down(C, dC, (size_t)M * N * es);
  return st.finish();
}

int gemv_host(int dtype, int32_t M, int32_t N, double alpha, const void* A, const void* x, double beta, void* y) {
  if (M < 0 || N < 0 || !A || !x || !y) return fail(AMC_ERR_INVALID, "gemv: bad arguments");
  size_t es = dtype_size(dtype);
  Staging st(default_stream());
  void* dA = st.up(A, (size_t)M * N * es);
  void* dx = st.up(x, (size_t)N * es);
  void* dy = st.up(beta != 0.0 ? y : nullptr, (size_t)M * es);
  if (st.rc) return st.finish();
  GemmArgs g;
  memset(&g, 0, sizeof g);
  g.M = M; g.N = 1; g.K = N;
  g.A = dA; g.a_dtype = dtype; g.sa0 = N; g.sa1 = 1;
  g.B = dx; g.b_dtype = dtype; g.sb0 = 1; g.sb1 = 0;
  g.C = dy; g.c_dtype = dtype;
  g.alpha = alpha; g.beta = beta;
  void* scratch = nullptr;
  if (size_t sb = gemm_scratch_bytes(g)) scratch = st.up(nullptr, sb);
  if (st.rc) return st.finish();
  int rc = launch_gemm_scratch(g, scratch, st.s);
  if (rc) { st.rc = rc; return st.finish(); }
  st.down(y, dy, (size_t)M * es);
  return st.finish();
}

int dot_host(int dtype, int32_t N, const void* x, const void* y, void* out) {
  if (N < 0 || !x || !y || !out) return fail(AMC_ERR_INVALID, "dot: bad arguments");
  size_t es = dtype_size(dtype);
  Staging st(default_stream());
  void* dx = st.up(x, (size_t)N * es);
  void* dy = st.up(y, (size_t)N * es);
  void* dr = st.up(nullptr, es);
  if (st.rc) return st.finish();
  GemmArgs g;
  memset(&g, 0, sizeof g);
  g.M = 1; g.N = 1; g.K = N;
  g.A = dx; g.a_dtype = dtype; g.sa0 = 0; g.sa1 = 1;
  g.B = dy; g.b_dtype = dtype; g.sb0 = 1; g.sb1 = 0;
  g.C = dr; g.c_dtype = dtype;
  g.alpha = 1.0; g.beta = 0.0;
  void* scratch = nullptr;
  if (size_t sb = gemm_scratch_bytes(g)) scratch = st.up(nullptr, sb);
  if (st.rc) return st.finish();
  int rc = launch_gemm_scratch(g, scratch, st.s);
  if (rc) { st.rc = rc; return st.finish(); }
  st.down(out, dr, es);
  return st.finish();
}

int axpy_host(int dtype, int32_t N, double alpha, const void* x, void* y) {
  if (N < 0 || !x || !y) return fail(AMC_ERR_INVALID, "axpy: bad arguments");
  size_t es = dtype_size(dtype);
  Staging st(default_stream());
  void* dx = st.up(x, (size_t)N * es);
  void* dy = st.up(y, (size_t)N * es);
  if (st.rc) return st.finish();
  if (N) {
    k_axpy<<<(unsigned)((N + 255) / 256), 256, 0, st.s>>>(N, alpha, dx, dy, dtype);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) { st.rc = cuda_fail(e, "k_axpy"); return st.finish(); }
  }
  st.down(y, dy, (size_t)N * es);
  return st.finish();
}
}  // namespace

}  // namespace amc

using namespace amc;

extern "C" {

int amc_blas_dgemm(int32_t M, int32_t N, int32_t K, double alpha, const double* A, const double* B, double beta, double* C) {
  return gemm_host(AMC_F64, M, N, K, alpha, A, K, 0, B, N, 0, beta, C);
}
int amc_blas_sgemm(int32_t M, int32_t N, int32_t K, float alpha, const float* A, const float* B, float beta, float* C) {
  return gemm_host(AMC_F32, M, N, K, alpha, A, K, 0, B, N, 0, beta, C);
}
int amc_blas_dgemm_strided(int32_t M, int32_t N, int32_t K, double alpha, const double* A, int32_t lda, int32_t transA,
                           const double* B, int32_t ldb, int32_t transB, double beta, double* C) {
  return gemm_host(AMC_F64, M, N, K, alpha, A, lda, transA, B, ldb, transB, beta, C);
}
int amc_blas_sgemm_strided(int32_t M, int32_t N, int32_t K, float alpha, const float* A, int32_t lda, int32_t transA,
                           const float* B, int32_t ldb, int32_t transB, float beta, float* C) {
  return gemm_host(AMC_F32, M, N, K, alpha, A, lda, transA, B, ldb, transB, beta, C);
}
int amc_blas_dgemv(int32_t M, int32_t N, double alpha, const double* A, const double* x, double beta, double* y) {
  return gemv_host(AMC_F64, M, N, alpha, A, x, beta, y);
}
int amc_blas_sgemv(int32_t M, int32_t N, float alpha, const float* A, const float* x, float beta, float* y) {
  return gemv_host(AMC_F32, M, N, alpha, A, x, beta, y);
}
int amc_blas_ddot(int32_t N, const double* x, const double* y, double* out) { return dot_host(AMC_F64, N, x, y, out); }
int amc_blas_sdot(int32_t N, const float* x, const float* y, float* out) { return dot_host(AMC_F32, N, x, y, out); }
int amc_blas_daxpy(int32_t N, double alpha, const double* x, double* y) { return axpy_host(AMC_F64, N, alpha, x, y); }
int amc_blas_saxpy(int32_t N, float alpha, const float* x, float* y) { return axpy_host(AMC_F32, N, alpha, x, y); }

}  // extern "C"
