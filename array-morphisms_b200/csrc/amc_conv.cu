// 2-D convolution entry points (NCHW, f32) with the reference's arithmetic:
//   forward  = reshape(W2d . im2col(X))          (execute-conv2d-blas, realization.scm:166-252)
//   dgrad    = col2im(W2d^T . dY)                (execute-col2im-batched, :1196-1268)
//   wgrad    = sum_n dY_n . im2col(X_n)^T        (batch-reduce of per-sample GEMMs)
// Direct kernels: one thread per output element, GEMM sums in double in
// ascending reduction order and rounded to f32 where the reference stores
// (the GEMM result; then col2im's running f32 sum over (kh, kw); then the
// batch sum over n).  These match the reference compositions bit for bit and
// serve every shape; the tensor-core kernels take the shapes they support.
#include "amc_internal.h"

namespace amc {

struct ConvShape {
  int N, C, H, W, K, KH, KW, SH, SW, PH, PW, OH, OW;
};

__global__ void k_conv_fwd_direct(const float* __restrict__ X, const float* __restrict__ Wt, float* __restrict__ Y, ConvShape s) {
  long long total = (long long)s.N * s.K * s.OH * s.OW;
  long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= total) return;
  int ow = (int)(i % s.OW), oh = (int)((i / s.OW) % s.OH), k = (int)((i / ((long long)s.OW * s.OH)) % s.K);
  long long n = i / ((long long)s.OW * s.OH * s.K);
  double acc = 0.0;
  for (int c = 0; c < s.C; ++c)
    for (int kh = 0; kh < s.KH; ++kh)
      for (int kw = 0; kw < s.KW; ++kw) {
        int ih = oh * s.SH + kh - s.PH, iw = ow * s.SW + kw - s.PW;
        double x = (ih >= 0 && ih < s.H && iw >= 0 && iw < s.W) ? (double)__ldg(X + ((n * s.C + c) * s.H + ih) * s.W + iw) : 0.0;
        acc = __dadd_rn(acc, __dmul_rn((double)__ldg(Wt + ((long long)(k * s.C + c) * s.KH + kh) * s.KW + kw), x));
      }
  Y[i] = __double2float_rn(acc);
}

__global__ void k_conv_dgrad_direct(const float* __restrict__ dY, const float* __restrict__ Wt, float* __restrict__ dX, ConvShape s) {
  long long total = (long long)s.N * s.C * s.H * s.W;
  long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= total) return;
  int w = (int)(i % s.W), h = (int)((i / s.W) % s.H), c = (int)((i / ((long long)s.W * s.H)) % s.C);
  long long n = i / ((long long)s.W * s.H * s.C);
  float acc = 0.f;
  for (int kh = 0; kh < s.KH; ++kh) {
    int th = h + s.PH - kh;
    if (th < 0 || th % s.SH) continue;
    int oh = th / s.SH;
    if (oh >= s.OH) continue;
    for (int kw = 0; kw < s.KW; ++kw) {
      int tw = w + s.PW - kw;
      if (tw < 0 || tw % s.SW) continue;
      int ow = tw / s.SW;
      if (ow >= s.OW) continue;
      double g = 0.0;  // col[(c,kh,kw), (oh,ow)] = sum_k W[k,(c,kh,kw)] dY[k,(oh,ow)]
      for (int k = 0; k < s.K; ++k)
        g = __dadd_rn(g, __dmul_rn((double)__ldg(Wt + ((long long)(k * s.C + c) * s.KH + kh) * s.KW + kw),
                                   (double)__ldg(dY + ((n * s.K + k) * s.OH + oh) * s.OW + ow)));
      acc = __double2float_rn(__dadd_rn((double)acc, (double)__double2float_rn(g)));
    }
  }
  dX[i] = acc;
}

__global__ void k_conv_wgrad_direct(const float* __restrict__ X, const float* __restrict__ dY, float* __restrict__ dW, ConvShape s) {
  long long total = (long long)s.K * s.C * s.KH * s.KW;
  long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= total) return;
  int kw = (int)(i % s.KW), kh = (int)((i / s.KW) % s.KH), c = (int)((i / (s.KW * s.KH)) % s.C);
  int k = (int)(i / ((long long)s.KW * s.KH * s.C));
  float acc = 0.f;
  for (int n = 0; n < s.N; ++n) {
    double g = 0.0;
    for (int oh = 0; oh < s.OH; ++oh)
      for (int ow = 0; ow < s.OW; ++ow) {
        int ih = oh * s.SH + kh - s.PH, iw = ow * s.SW + kw - s.PW;
        double x = (ih >= 0 && ih < s.H && iw >= 0 && iw < s.W) ? (double)__ldg(X + (((long long)n * s.C + c) * s.H + ih) * s.W + iw) : 0.0;
        g = __dadd_rn(g, __dmul_rn((double)__ldg(dY + (((long long)n * s.K + k) * s.OH + oh) * s.OW + ow), x));
      }
    acc = __double2float_rn(__dadd_rn((double)acc, (double)__double2float_rn(g)));
  }
  dW[i] = acc;
}

static int conv_shape(ConvShape& s, int32_t N, int32_t C, int32_t H, int32_t W, int32_t K, int32_t KH, int32_t KW,
                      int32_t SH, int32_t SW, int32_t PH, int32_t PW) {
  if (N < 0 || C <= 0 || H <= 0 || W <= 0 || K <= 0 || KH <= 0 || KW <= 0 || SH <= 0 || SW <= 0 || PH < 0 || PW < 0)
    return fail(AMC_ERR_INVALID, "conv2d: bad shape");
  s = ConvShape{N, C, H, W, K, KH, KW, SH, SW, PH, PW, 1 + (H + 2 * PH - KH) / SH, 1 + (W + 2 * PW - KW) / SW};
  if (s.OH <= 0 || s.OW <= 0) return fail(AMC_ERR_INVALID, "conv2d: kernel larger than the padded image");
  return AMC_OK;
}

int conv_fwd_tc(const float* X, const float* W, float* Y, const ConvShape& s, cudaStream_t st, bool* handled);
int conv_dgrad_tc(const float* dY, const float* W, float* dX, const ConvShape& s, cudaStream_t st, bool* handled);
int conv_wgrad_tc(const float* X, const float* dY, float* dW, const ConvShape& s, cudaStream_t st, bool* handled);


}  // namespace amc

using namespace amc;

extern "C" {

int amc_conv2d_fwd_f32(const float* X, const float* W, float* Y, int32_t N, int32_t C, int32_t H, int32_t Wd, int32_t K,
                       int32_t KH, int32_t KW, int32_t SH, int32_t SW, int32_t PH, int32_t PW, void* stream) {
  ConvShape s;
  int rc = conv_shape(s, N, C, H, Wd, K, KH, KW, SH, SW, PH, PW);
  if (rc) return rc;
  if (!X || !W || !Y) return fail(AMC_ERR_INVALID, "conv2d: null pointer");
  if (fault_injected("launch")) return fail(AMC_ERR_INJECTED, "conv2d: injected launch failure (AMC_FAULT=launch)");
  cudaStream_t st = pick_stream(stream);
  bool handled = false;
  rc = conv_fwd_tc(X, W, Y, s, st, &handled);
  if (rc || handled) return rc;
  long long total = (long long)N * K * s.OH * s.OW;
  if (total) k_conv_fwd_direct<<<(unsigned)((total + 255) / 256), 256, 0, st>>>(X, W, Y, s);
  AMC_CUDA(cudaGetLastError());
  return AMC_OK;
}

int amc_conv2d_dgrad_f32(const float* dY, const float* W, float* dX, int32_t N, int32_t C, int32_t H, int32_t Wd,
                         int32_t K, int32_t KH, int32_t KW, int32_t SH, int32_t SW, int32_t PH, int32_t PW, void* stream) {
  ConvShape s;
  int rc = conv_shape(s, N, C, H, Wd, K, KH, KW, SH, SW, PH, PW);
  if (rc) return rc;
  if (!dY || !W || !dX) return fail(AMC_ERR_INVALID, "conv2d: null pointer");
  cudaStream_t st = pick_stream(stream);
  bool handled = false;
  rc = conv_dgrad_tc(dY, W, dX, s, st, &handled);
  if (rc || handled) return rc;
  long long total = (long long)N * C * H * Wd;
  if (total) k_conv_dgrad_direct<<<(unsigned)((total + 255) / 256), 256, 0, st>>>(dY, W, dX, s);
  AMC_CUDA(cudaGetLastError());
  return AMC_OK;
}

int amc_conv2d_wgrad_f32(const float* X, const float* dY, float* dW, int32_t N, int32_t C, int32_t H, int32_t Wd,
                         int32_t K, int32_t KH, int32_t KW, int32_t SH, int32_t SW, int32_t PH, int32_t PW, void* stream) {
  ConvShape s;
  int rc = conv_shape(s, N, C, H, Wd, K, KH, KW, SH, SW, PH, PW);
  if (rc) return rc;
  if (!X || !dY || !dW) return fail(AMC_ERR_INVALID, "conv2d: null pointer");
  cudaStream_t st = pick_stream(stream);
  bool handled = false;
  rc = conv_wgrad_tc(X, dY, dW, s, st, &handled);
  if (rc || handled) return rc;
  long long total = (long long)K * C * KH * KW;
  if (total) k_conv_wgrad_direct<<<(unsigned)((total + 255) / 256), 256, 0, st>>>(X, dY, dW, s);
  AMC_CUDA(cudaGetLastError());
  return AMC_OK;
}

}  // extern "C"
