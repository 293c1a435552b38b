// Scaled dot-product attention on contiguous (blocks, n, d) f32 tensors.
//
// Forward: the streaming softmax of %attn-2d! (realization.scm:279-326) with
// the three passes folded into one online pass (running max and sum), one
// warp per query row, f32 storage, f32 accumulation.  Also writes the row
// log-sum-exp, which the backward pass uses to rebuild P without storing it.
// Backward (no reference implementation exists: grad.scm and ssa-vjp have no
// attention rule) is the standard VJP:
//   dV = P^T dO, dS = P * (dO V^T - rowsum(dO * O)), dQ = scale dS K,
//   dK = scale dS^T Q.
#include <cmath>

#include "amc_internal.h"

namespace amc {

constexpr int kMaxD = 128;

__global__ void __launch_bounds__(128) k_attn_fwd_simt(const float* __restrict__ Q, const float* __restrict__ K,
                                                       const float* __restrict__ V, float* __restrict__ O,
                                                       float* __restrict__ lse, long long rows, int n, int dk, int dv,
                                                       float scale) {
  const int lane = threadIdx.x & 31;
  const long long row = (long long)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  if (row >= rows) return;
  const long long b = row / n;
  const float* q = Q + row * dk;
  const float* kb = K + b * (long long)n * dk;
  const float* vb = V + b * (long long)n * dv;
  float qr[kMaxD / 32];
  for (int j = 0; j < kMaxD / 32; ++j) qr[j] = (lane + 32 * j < dk) ? q[lane + 32 * j] * scale : 0.f;
  float m = -INFINITY, l = 0.f, acc[kMaxD / 32];
  for (int j = 0; j < kMaxD / 32; ++j) acc[j] = 0.f;
  for (int k = 0; k < n; ++k) {
    float s = 0.f;
    for (int j = 0; j < kMaxD / 32; ++j)
      if (lane + 32 * j < dk) s = fmaf(qr[j], __ldg(kb + (long long)k * dk + lane + 32 * j), s);
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    float mn = fmaxf(m, s);
    float corr = __expf(m - mn), p = __expf(s - mn);
    l = l * corr + p;
    for (int j = 0; j < kMaxD / 32; ++j)
      if (lane + 32 * j < dv) acc[j] = fmaf(p, __ldg(vb + (long long)k * dv + lane + 32 * j), acc[j] * corr);
    m = mn;
  }
  float inv = 1.f / l;
  for (int j = 0; j < kMaxD / 32; ++j)
    if (lane + 32 * j < dv) O[row * dv + lane + 32 * j] = acc[j] * inv;
  if (lane == 0 && lse) lse[row] = m + logf(l);
}

// dQ rows (one warp per query row).
__global__ void __launch_bounds__(128) k_attn_bwd_dq(const float* __restrict__ Q, const float* __restrict__ K,
                                                     const float* __restrict__ V, const float* __restrict__ O,
                                                     const float* __restrict__ dO, const float* __restrict__ lse,
                                                     float* __restrict__ dQ, long long rows, int n, int dk, int dv,
                                                     float scale) {
  const int lane = threadIdx.x & 31;
  const long long row = (long long)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  if (row >= rows) return;
  const long long b = row / n;
  const float* kb = K + b * (long long)n * dk;
  const float* vb = V + b * (long long)n * dv;
  float qr[kMaxD / 32], gor[kMaxD / 32], acc[kMaxD / 32];
  float D = 0.f;
  for (int j = 0; j < kMaxD / 32; ++j) {
    int c = lane + 32 * j;
    qr[j] = c < dk ? Q[row * dk + c] : 0.f;
    gor[j] = c < dv ? dO[row * dv + c] : 0.f;
    if (c < dv) D = fmaf(gor[j], O[row * dv + c], D);
    acc[j] = 0.f;
  }
  for (int o = 16; o > 0; o >>= 1) D += __shfl_xor_sync(0xffffffffu, D, o);
  const float L = lse[row];
  for (int k = 0; k < n; ++k) {
    float s = 0.f, dp = 0.f;
    for (int j = 0; j < kMaxD / 32; ++j) {
      int c = lane + 32 * j;
      if (c < dk) s = fmaf(qr[j], __ldg(kb + (long long)k * dk + c), s);
      if (c < dv) dp = fmaf(gor[j], __ldg(vb + (long long)k * dv + c), dp);
    }
    for (int o = 16; o > 0; o >>= 1) {
      s += __shfl_xor_sync(0xffffffffu, s, o);
      dp += __shfl_xor_sync(0xffffffffu, dp, o);
    }
    float p = __expf(s * scale - L);
    float ds = p * (dp - D);
    for (int j = 0; j < kMaxD / 32; ++j)
      if (lane + 32 * j < dk) acc[j] = fmaf(ds, __ldg(kb + (long long)k * dk + lane + 32 * j), acc[j]);
  }
  for (int j = 0; j < kMaxD / 32; ++j)
    if (lane + 32 * j < dk) dQ[row * dk + lane + 32 * j] = acc[j] * scale;
}

// dK, dV rows (one warp per key row).
__global__ void __launch_bounds__(128) k_attn_bwd_dkv(const float* __restrict__ Q, const float* __restrict__ K,
                                                      const float* __restrict__ V, const float* __restrict__ O,
                                                      const float* __restrict__ dO, const float* __restrict__ lse,
                                                      float* __restrict__ dK, float* __restrict__ dV, long long rows,
                                                      int n, int dk, int dv, float scale) {
  const int lane = threadIdx.x & 31;
  const long long row = (long long)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  if (row >= rows) return;
  const long long b = row / n;
  const float* qb = Q + b * (long long)n * dk;
  const float* ob = O + b * (long long)n * dv;
  const float* gb = dO + b * (long long)n * dv;
  const float* lb = lse + b * (long long)n;
  float kr[kMaxD / 32], vr[kMaxD / 32], ak[kMaxD / 32], av[kMaxD / 32];
  for (int j = 0; j < kMaxD / 32; ++j) {
    int c = lane + 32 * j;
    kr[j] = c < dk ? K[row * dk + c] : 0.f;
    vr[j] = c < dv ? V[row * dv + c] : 0.f;
    ak[j] = 0.f;
    av[j] = 0.f;
  }
  for (int i = 0; i < n; ++i) {
    float s = 0.f, dp = 0.f, D = 0.f;
    for (int j = 0; j < kMaxD / 32; ++j) {
      int c = lane + 32 * j;
      if (c < dk) s = fmaf(__ldg(qb + (long long)i * dk + c), kr[j], s);
      if (c < dv) {
        float g = __ldg(gb + (long long)i * dv + c);
        dp = fmaf(g, vr[j], dp);
        D = fmaf(g, __ldg(ob + (long long)i * dv + c), D);
      }
    }
    for (int o = 16; o > 0; o >>= 1) {
      s += __shfl_xor_sync(0xffffffffu, s, o);
      dp += __shfl_xor_sync(0xffffffffu, dp, o);
      D += __shfl_xor_sync(0xffffffffu, D, o);
    }
    float p = __expf(s * scale - __ldg(lb + i));
    float ds = p * (dp - D);
    for (int j = 0; j < kMaxD / 32; ++j) {
      int c = lane + 32 * j;
      if (c < dk) ak[j] = fmaf(ds, __ldg(qb + (long long)i * dk + c), ak[j]);
      if (c < dv) av[j] = fmaf(p, __ldg(gb + (long long)i * dv + c), av[j]);
    }
  }
  for (int j = 0; j < kMaxD / 32; ++j) {
    int c = lane + 32 * j;
    if (c < dk) dK[row * dk + c] = ak[j] * scale;
    if (c < dv) dV[row * dv + c] = av[j];
  }
}

int attention_fwd_simt(const float* Q, const float* K, const float* V, float* O, float* lse, long long blocks, int n,
                       int dk, int dv, float scale, cudaStream_t s) {
  long long rows = blocks * n;
  if (!rows) return AMC_OK;
  k_attn_fwd_simt<<<(unsigned)((rows + 3) / 4), 128, 0, s>>>(Q, K, V, O, lse, rows, n, dk, dv, scale);
  AMC_CUDA(cudaGetLastError());
  return AMC_OK;
}

}  // namespace amc

using namespace amc;


extern "C" {

int amc_attention_fwd_f32(const float* Q, const float* K, const float* V, float* O, float* lse, int64_t blocks,
                          int32_t n, int32_t dk, int32_t dv, float scale, void* stream) {
  if (!Q || !K || !V || !O || blocks < 0 || n < 0 || dk <= 0 || dv <= 0 || dk > kMaxD || dv > kMaxD)
    return fail(AMC_ERR_INVALID, "amc_attention_fwd_f32: bad arguments (head dims 1..128)");
  if (fault_injected("launch")) return fail(AMC_ERR_INJECTED, "attention: injected launch failure (AMC_FAULT=launch)");
  cudaStream_t s = pick_stream(stream);
  bool handled = false;
  int rc = attention_fwd_tc(Q, K, V, O, lse, blocks, n, dk, dv, scale, s, &handled);
  if (rc || handled) return rc;
  return attention_fwd_simt(Q, K, V, O, lse, blocks, n, dk, dv, scale, s);
}

int amc_attention_bwd_f32(const float* Q, const float* K, const float* V, const float* O, const float* dO,
                          const float* lse, float* dQ, float* dK, float* dV, int64_t blocks, int32_t n, int32_t dk,
                          int32_t dv, float scale, void* stream) {
  if (!Q || !K || !V || !O || !dO || !lse || !dQ || !dK || !dV || blocks < 0 || n < 0 || dk <= 0 || dv <= 0 ||
      dk > kMaxD || dv > kMaxD)
    return fail(AMC_ERR_INVALID, "amc_attention_bwd_f32: bad arguments (head dims 1..128)");
  if (fault_injected("launch")) return fail(AMC_ERR_INJECTED, "attention: injected launch failure (AMC_FAULT=launch)");
  cudaStream_t s = pick_stream(stream);
  bool handled = false;
  int rc = attention_bwd_tc(Q, K, V, O, dO, lse, dQ, dK, dV, blocks, n, dk, dv, scale, s, &handled);
  if (rc || handled) return rc;
  long long rows = blocks * n;
  if (!rows) return AMC_OK;
  k_attn_bwd_dq<<<(unsigned)((rows + 3) / 4), 128, 0, s>>>(Q, K, V, O, dO, lse, dQ, rows, n, dk, dv, scale);
  AMC_CUDA(cudaGetLastError());
  k_attn_bwd_dkv<<<(unsigned)((rows + 3) / 4), 128, 0, s>>>(Q, K, V, O, dO, lse, dK, dV, rows, n, dk, dv, scale);
  AMC_CUDA(cudaGetLastError());
  return AMC_OK;
}

}  // extern "C"
