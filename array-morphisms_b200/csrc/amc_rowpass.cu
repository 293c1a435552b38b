// Row passes over a row-major matrix X (rows x d, unit stride along d): the
// matrix-vector products of the BLAS layer at sizes where one CTA per output
// tile cannot fill the GPU, and the linear model's GEMV pair in ONE read of X.
//
//   FWD        p_i = sum_k X[i,k] w[k]            (GEMV; blas-exec.scm:735-793)
//   ACC        out[k] = sum_i X[i,k] e_i           (X^T e: the transposed GEMV,
//                                                   blas-exec.scm:666-731 with transA)
//   FWD + ACC  e_i = prog(p_i, row-aligned leaves at i): the gradient GEMV of
//              ssa-vjp's matmul rule (ssa.scm:922-940) over an element-wise
//              function of the forward GEMV's result, the MSE step of the
//              SSA replay (ssa.scm:1519-1654) without a second read of X.
//
// The reference accumulates each output sequentially in double
// (blas-exec.scm:405-458).  Here a warp owns contiguous rows: p_i is a
// lane-strided fma sum finished by a fixed shuffle tree, X^T e accumulates
// per warp in row order, warps combine in index order and CTA partials in a
// fixed 8-group order.  Results are deterministic on a given GPU and agree
// with the sequential order to double rounding error; the planner sends only
// large shapes here, so the small known-answer cases keep the reference's
// order bit for bit through k_gemm.
#include <cstring>

#include "amc_internal.h"

namespace amc {

namespace {

constexpr int kRowBlock = 256;
constexpr int kRowWarps = kRowBlock / 32;
constexpr unsigned kFull = 0xffffffffu;

__device__ __forceinline__ double ld_any(const void* p, int dtype, long long k) {
  return dtype == AMC_F32 ? (double)__ldg((const float*)p + k) : __ldg((const double*)p + k);
}
__device__ __forceinline__ double ld_stream(const float* p) { return (double)__ldcs(p); }
__device__ __forceinline__ double ld_stream(const double* p) { return __ldcs(p); }

__device__ __forceinline__ double round_to(int dtype, double v) {
  return dtype == AMC_F32 ? (double)__double2float_rn(v) : v;
}

__device__ __forceinline__ void store_to(void* p, int dtype, long long k, double v) {
  if (dtype == AMC_F32) ((float*)p)[k] = __double2float_rn(v);
  else ((double*)p)[k] = v;
}

// The row program on leaf values already in registers (every value a
// double; the program is all-float).
__device__ __forceinline__ double eval_row(const DProg& P, const double* lv) {
  double st[AMC_STACK_MAX];
  int sp = 0;
  for (int pc = 0; pc < P.n; ++pc) {
    const amc_insn I = P.code[pc];
    switch (I.op) {
      case AMC_OP_LOAD: st[sp++] = lv[I.a]; break;
      case AMC_OP_CONST: st[sp++] = I.imm; break;
      case AMC_OP_CVT: st[sp - 1] = round_to(I.a, st[sp - 1]); break;
      case AMC_OP_NEG: st[sp - 1] = -st[sp - 1]; break;
      case AMC_OP_ABS: st[sp - 1] = fabs(st[sp - 1]); break;
      case AMC_OP_FLOOR: st[sp - 1] = floor(st[sp - 1]); break;
      case AMC_OP_CEIL: st[sp - 1] = ceil(st[sp - 1]); break;
      case AMC_OP_SQRT: st[sp - 1] = sqrt(st[sp - 1]); break;
      case AMC_OP_EXP: st[sp - 1] = exp(st[sp - 1]); break;
      case AMC_OP_LOG: st[sp - 1] = log(st[sp - 1]); break;
      case AMC_OP_SIN: st[sp - 1] = sin(st[sp - 1]); break;
      case AMC_OP_COS: st[sp - 1] = cos(st[sp - 1]); break;
      case AMC_OP_TAN: st[sp - 1] = tan(st[sp - 1]); break;
      case AMC_OP_RELU: st[sp - 1] = st[sp - 1] > 0.0 ? st[sp - 1] : 0.0; break;
      case AMC_OP_SIGMOID: st[sp - 1] = __ddiv_rn(1.0, __dadd_rn(1.0, exp(-st[sp - 1]))); break;
      case AMC_OP_TANH: {
        double e2 = exp(__dmul_rn(2.0, st[sp - 1]));
        st[sp - 1] = __ddiv_rn(__dsub_rn(e2, 1.0), __dadd_rn(e2, 1.0));
      } break;
      default: {
        const double x = st[sp - 2], y = st[sp - 1];
        double r;
        switch (I.op) {
          case AMC_OP_ADD: r = __dadd_rn(x, y); break;
          case AMC_OP_SUB: r = __dsub_rn(x, y); break;
          case AMC_OP_MUL: r = __dmul_rn(x, y); break;
          case AMC_OP_DIV: r = __ddiv_rn(x, y); break;
          case AMC_OP_POW: r = pow(x, y); break;
          case AMC_OP_MAX: r = x > y ? x : y; break;
          case AMC_OP_MIN: r = x < y ? x : y; break;
          case AMC_OP_GT: r = (double)(x > y); break;
          case AMC_OP_LT: r = (double)(x < y); break;
          case AMC_OP_EQ: r = (double)(x == y); break;
          case AMC_OP_GE: r = (double)(x >= y); break;
          default: r = (double)(x <= y); break;
        }
        st[sp - 2] = r;
        --sp;
      }
    }
  }
  return st[0];
}

// Four lane-partial sums reduced across the warp in six shuffles: lane L ends
// with the full sum of value (L >> 3) & 3.  The order is fixed.
__device__ __forceinline__ double reduce4(double p0, double p1, double p2, double p3, int lane) {
  const bool hi = lane & 16;
  const double s0 = hi ? p0 : p2, s1 = hi ? p1 : p3;
  const double k0 = hi ? p2 : p0, k1 = hi ? p3 : p1;
  const double a0 = k0 + __shfl_xor_sync(kFull, s0, 16);
  const double a1 = k1 + __shfl_xor_sync(kFull, s1, 16);
  const bool b8 = lane & 8;
  double b = (b8 ? a1 : a0) + __shfl_xor_sync(kFull, b8 ? a0 : a1, 8);
  b += __shfl_xor_sync(kFull, b, 4);
  b += __shfl_xor_sync(kFull, b, 2);
  b += __shfl_xor_sync(kFull, b, 1);
  return b;
}

__device__ __forceinline__ double reduce1(double p) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) p += __shfl_xor_sync(kFull, p, o);
  return p;
}

// The forward product's stored value: alpha/beta as k_gemm applies them,
// rounded to the result dtype.
__device__ __forceinline__ double fwd_store(const RowPassArgs& a, long long i, double p) {
  double v = p;
  if (a.alpha != 1.0) v = __dmul_rn(a.alpha, v);
  if (a.beta != 0.0) v = __dadd_rn(v, __dmul_rn(a.beta, ld_any(a.r, a.r_dtype, i * a.sr)));
  v = round_to(a.r_dtype, v);
  if (a.r) store_to(a.r, a.r_dtype, i * a.sr, v);
  return v;
}

// Leaf values of row i (the forward product's leaf left for the caller).
__device__ __forceinline__ void load_row_leaves(const RowPassArgs& a, long long i, double* lv) {
#pragma unroll
  for (int l = 0; l < kMaxLeaves; ++l)
    if (l < a.nleaf && l != a.e_rleaf) lv[l] = ld_any(a.leaf[l].ptr, a.leaf[l].dtype, i * a.leaf[l].strides[0]);
}

// The row value e_i: the program over the row's leaves and the forward
// product (FWD), or the stored vector b (plain transposed GEMV).
template <bool FWD>
__device__ __forceinline__ double row_value(const RowPassArgs& a, long long i, double pr, double* lv) {
  if (FWD) {
    lv[a.e_rleaf] = pr;
    return eval_row(a.prog, lv);
  }
  return ld_any(a.b, a.b_dtype, i * a.sb);
}

template <typename T, int KPL, bool FWD, bool ACC>
__global__ void __launch_bounds__(kRowBlock) k_rowpass(const __grid_constant__ RowPassArgs a) {
  constexpr int D = 32 * KPL;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const long long gw = (long long)blockIdx.x * kRowWarps + warp, tw = (long long)gridDim.x * kRowWarps;
  const long long r0 = a.rows * gw / tw, r1 = a.rows * (gw + 1) / tw;
  const T* X = (const T*)a.X;
  double wv[KPL], acc[KPL];
#pragma unroll
  for (int j = 0; j < KPL; ++j) {
    wv[j] = FWD ? ld_any(a.w, a.w_dtype, (long long)(lane + 32 * j) * a.sw) : 0.0;
    acc[j] = 0.0;
  }
  const int q_own = (lane >> 3) & 3;
  const bool owner = (lane & 7) == 0;
  long long i = r0;
  for (; i + 4 <= r1; i += 4) {
    double x[4][KPL];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const T* px = X + (i + q) * a.ldx + lane;
#pragma unroll
      for (int j = 0; j < KPL; ++j) x[q][j] = ld_stream(px + 32 * j);
    }
    double lv[kMaxLeaves];
    if (ACC && FWD && owner) load_row_leaves(a, i + q_own, lv);
    double ev = 0.0;
    if (FWD) {
      double p[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        p[q] = 0.0;
#pragma unroll
        for (int j = 0; j < KPL; ++j) p[q] = fma(x[q][j], wv[j], p[q]);
      }
      const double s = reduce4(p[0], p[1], p[2], p[3], lane);
      if (owner) {
        const double pr = fwd_store(a, i + q_own, s);
        if (ACC) ev = row_value<true>(a, i + q_own, pr, lv);
      }
    } else if (owner) {
      ev = row_value<false>(a, i + q_own, 0.0, lv);
    }
    if (ACC) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const double e = __shfl_sync(kFull, ev, 8 * q);
#pragma unroll
        for (int j = 0; j < KPL; ++j) acc[j] = fma(x[q][j], e, acc[j]);
      }
    }
  }
  for (; i < r1; ++i) {
    double x[KPL];
    const T* px = X + i * a.ldx + lane;
#pragma unroll
    for (int j = 0; j < KPL; ++j) x[j] = ld_stream(px + 32 * j);
    double lv[kMaxLeaves];
    if (ACC && FWD && lane == 0) load_row_leaves(a, i, lv);
    double ev = 0.0;
    if (FWD) {
      double p = 0.0;
#pragma unroll
      for (int j = 0; j < KPL; ++j) p = fma(x[j], wv[j], p);
      p = reduce1(p);
      if (lane == 0) {
        const double pr = fwd_store(a, i, p);
        if (ACC) ev = row_value<true>(a, i, pr, lv);
      }
    } else if (lane == 0) {
      ev = row_value<false>(a, i, 0.0, lv);
    }
    if (ACC) {
      const double e = __shfl_sync(kFull, ev, 0);
#pragma unroll
      for (int j = 0; j < KPL; ++j) acc[j] = fma(x[j], e, acc[j]);
    }
  }
  if (ACC) {
    // the CTA's warps combined in index order
    __shared__ double sm[kRowWarps][D];
#pragma unroll
    for (int j = 0; j < KPL; ++j) sm[warp][lane + 32 * j] = acc[j];
    __syncthreads();
    for (int k = threadIdx.x; k < D; k += kRowBlock) {
      double s = 0.0;
#pragma unroll
      for (int ww = 0; ww < kRowWarps; ++ww) s += sm[ww][k];
      a.partials[(long long)blockIdx.x * D + k] = s;
    }
  }
}

// Any d <= 1024: one row at a time, lanes striding over the columns, the
// transposed product's accumulators in shared memory (one row per warp).
template <typename T, bool FWD, bool ACC>
__global__ void __launch_bounds__(kRowBlock) k_rowpass_any(const __grid_constant__ RowPassArgs a) {
  extern __shared__ double acc_sm[];   // [kRowWarps][d] when ACC
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, d = a.d;
  const long long gw = (long long)blockIdx.x * kRowWarps + warp, tw = (long long)gridDim.x * kRowWarps;
  const long long r0 = a.rows * gw / tw, r1 = a.rows * (gw + 1) / tw;
  const T* X = (const T*)a.X;
  double* acc = acc_sm + (size_t)warp * d;
  if (ACC)
    for (int k = lane; k < d; k += 32) acc[k] = 0.0;
  __syncwarp();
  for (long long i = r0; i < r1; ++i) {
    const T* px = X + i * a.ldx;
    double lv[kMaxLeaves];
    if (ACC && FWD && lane == 0) load_row_leaves(a, i, lv);
    double ev = 0.0;
    if (FWD) {
      double p = 0.0;
      for (int k = lane; k < d; k += 32) p = fma(ld_stream(px + k), ld_any(a.w, a.w_dtype, (long long)k * a.sw), p);
      p = reduce1(p);
      if (lane == 0) {
        const double pr = fwd_store(a, i, p);
        if (ACC) ev = row_value<true>(a, i, pr, lv);
      }
    } else if (lane == 0) {
      ev = row_value<false>(a, i, 0.0, lv);
    }
    if (ACC) {
      const double e = __shfl_sync(kFull, ev, 0);
      for (int k = lane; k < d; k += 32) acc[k] = fma((double)px[k], e, acc[k]);
    }
  }
  if (ACC) {
    __syncthreads();
    for (int k = threadIdx.x; k < d; k += kRowBlock) {
      double s = 0.0;
      for (int ww = 0; ww < kRowWarps; ++ww) s += acc_sm[(size_t)ww * d + k];
      a.partials[(long long)blockIdx.x * d + k] = s;
    }
  }
}

// Dot product partials: CTA b sums a contiguous K range, threads strided
// within it, then a fixed shuffle tree and the warps in index order.
template <typename TA, typename TB>
__global__ void __launch_bounds__(kRowBlock) k_dot_partials(const TA* __restrict__ x, long long sx,
                                                            const TB* __restrict__ y, long long sy, long long K,
                                                            double* __restrict__ partials) {
  const long long b0 = K * blockIdx.x / gridDim.x, b1 = K * (blockIdx.x + 1) / gridDim.x;
  double s = 0.0;
  for (long long k = b0 + threadIdx.x; k < b1; k += kRowBlock)
    s = fma((double)__ldcs(x + k * sx), (double)__ldcs(y + k * sy), s);
  s = reduce1(s);
  __shared__ double ws[kRowWarps];
  if ((threadIdx.x & 31) == 0) ws[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    double t = 0.0;
#pragma unroll
    for (int w = 0; w < kRowWarps; ++w) t += ws[w];
    partials[blockIdx.x] = t;
  }
}

// out[k] = sum of the n partial rows, in a fixed order: a CTA takes 32
// columns and 8 groups of rows; group g adds rows g, g+8, ... ascending, then
// the 8 group sums are added pairwise in index order.  alpha/beta as k_gemm.
__global__ void __launch_bounds__(256) k_rowpass_reduce(const double* __restrict__ partials, int n, int d, void* out,
                                                        int out_dtype, long long sout, double alpha, double beta) {
  __shared__ double red[8][33];
  const int l = threadIdx.x & 31, g = threadIdx.x >> 5;
  const int k = blockIdx.x * 32 + l;
  double s = 0.0;
  if (k < d)
    for (int b = g; b < n; b += 8) s += __ldg(partials + (long long)b * d + k);
  red[g][l] = s;
  __syncthreads();
  if (g == 0 && k < d) {
    double v = ((red[0][l] + red[1][l]) + (red[2][l] + red[3][l])) + ((red[4][l] + red[5][l]) + (red[6][l] + red[7][l]));
    if (alpha != 1.0) v = __dmul_rn(alpha, v);
    if (beta != 0.0) v = __dadd_rn(v, __dmul_rn(beta, ld_any(out, out_dtype, k * sout)));
    store_to(out, out_dtype, k * sout, v);
  }
}

std::atomic<uint64_t> g_any_smem_done[2][3];

template <typename T, bool FWD, bool ACC>
int launch_any(const RowPassArgs& a, int grid, cudaStream_t s) {
  const size_t sm = ACC ? (size_t)kRowWarps * a.d * sizeof(double) : 0;
  if (sm > 48 * 1024) {
    const int slot = FWD ? (ACC ? 0 : 1) : 2;
    int rc = smem_attr_once(k_rowpass_any<T, FWD, ACC>, (int)sm, g_any_smem_done[sizeof(T) == 8][slot]);
    if (rc) return rc;
  }
  k_rowpass_any<T, FWD, ACC><<<grid, kRowBlock, sm, s>>>(a);
  return AMC_OK;
}

template <typename T, bool FWD, bool ACC>
int launch_mode(const RowPassArgs& a, int grid, cudaStream_t s) {
  switch (a.d) {
    case 32: k_rowpass<T, 1, FWD, ACC><<<grid, kRowBlock, 0, s>>>(a); return AMC_OK;
    case 64: k_rowpass<T, 2, FWD, ACC><<<grid, kRowBlock, 0, s>>>(a); return AMC_OK;
    case 128: k_rowpass<T, 4, FWD, ACC><<<grid, kRowBlock, 0, s>>>(a); return AMC_OK;
    case 256: k_rowpass<T, 8, FWD, ACC><<<grid, kRowBlock, 0, s>>>(a); return AMC_OK;
    default: return launch_any<T, FWD, ACC>(a, grid, s);
  }
}

template <typename T>
int launch_typed(const RowPassArgs& a, int grid, cudaStream_t s) {
  if (a.fwd && a.acc) return launch_mode<T, true, true>(a, grid, s);
  if (a.fwd) return launch_mode<T, true, false>(a, grid, s);
  return launch_mode<T, false, true>(a, grid, s);
}

template <typename TA>
int launch_dot_a(const RowPassArgs& a, int grid, cudaStream_t s) {
  const TA* x = (const TA*)a.X;
  if (a.b_dtype == AMC_F32) k_dot_partials<TA, float><<<grid, kRowBlock, 0, s>>>(x, a.ldx, (const float*)a.b, a.sb, a.rows, a.partials);
  else k_dot_partials<TA, double><<<grid, kRowBlock, 0, s>>>(x, a.ldx, (const double*)a.b, a.sb, a.rows, a.partials);
  return AMC_OK;
}

}  // namespace

int rowpass_grid(int64_t rows) {
  long long g = (long long)num_sms() * 4;
  long long need = (rows + 31) / 32;   // at least 32 rows per CTA
  if (need < g) g = need;
  return (int)(g < 1 ? 1 : g);
}

size_t rowpass_scratch_bytes(const RowPassArgs& a) {
  if (a.dot) return (size_t)rowpass_grid(a.rows) * sizeof(double);
  if (!a.acc) return 0;
  return (size_t)rowpass_grid(a.rows) * (size_t)a.d * sizeof(double);
}

int launch_rowpass(const RowPassArgs& a, cudaStream_t s) {
  if (a.rows < 0 || a.d < 1 || a.d > kRowPassMaxD || (!a.fwd && !a.acc && !a.dot))
    return fail(AMC_ERR_INVALID, "row pass: bad shape");
  if ((a.acc || a.dot) && !a.partials) return fail(AMC_ERR_INVALID, "row pass: no scratch for the partial sums");
  if (a.fwd && a.acc && (a.e_rleaf < 0 || a.e_rleaf >= a.nleaf || a.nleaf > kMaxLeaves))
    return fail(AMC_ERR_INVALID, "row pass: the row program does not read the forward product");
  if (fault_injected("launch")) return fail(AMC_ERR_INJECTED, "row pass: injected launch failure (AMC_FAULT=launch)");
  const int grid = rowpass_grid(a.rows);
  if (a.rows == 0) {
    // an empty contraction: every output is 0 (then alpha/beta)
    if (a.acc || a.dot) {
      AMC_CUDA(cudaMemsetAsync(a.partials, 0, rowpass_scratch_bytes(a), s));
      k_rowpass_reduce<<<(a.d + 31) / 32, 256, 0, s>>>(a.partials, 1, a.dot ? 1 : a.d, a.out, a.out_dtype, a.sout,
                                                       a.alpha, a.beta);
      AMC_CUDA(cudaGetLastError());
    }
    return AMC_OK;
  }
  int rc;
  if (a.dot) rc = a.x_dtype == AMC_F32 ? launch_dot_a<float>(a, grid, s) : launch_dot_a<double>(a, grid, s);
  else rc = a.x_dtype == AMC_F32 ? launch_typed<float>(a, grid, s) : launch_typed<double>(a, grid, s);
  if (rc) return rc;
  AMC_CUDA(cudaGetLastError());
  if (a.acc || a.dot) {
    const int d = a.dot ? 1 : a.d;
    k_rowpass_reduce<<<(d + 31) / 32, 256, 0, s>>>(a.partials, grid, d, a.out, a.out_dtype, a.sout, a.alpha, a.beta);
    AMC_CUDA(cudaGetLastError());
  }
  return AMC_OK;
}

int rowpass_launches(const RowPassArgs& a) { return (a.acc || a.dot) ? 2 : 1; }

// The matrix-vector shapes of a GEMM (N == 1) that the row passes take:
// a GEMV over row-contiguous A with K <= 1024, a transposed GEMV (A
// contiguous along M) with M <= 1024, and a dot product, each only when the
// contraction is large (see kRowPassMin*).  Smaller ones stay on k_gemm,
// which keeps the reference's sequential order bit for bit.
bool gemm_as_rowpass(const GemmArgs& g, RowPassArgs& r) {
  if (g.N != 1 || g.M < 1 || g.K < 1) return false;
  if (!dtype_float(g.a_dtype) || !dtype_float(g.b_dtype) || !dtype_float(g.c_dtype)) return false;
  memset(&r, 0, sizeof r);
  r.alpha = g.alpha;
  r.beta = g.beta;
  if (g.M == 1) {
    if (g.K < kRowPassMinDot) return false;
    r.dot = 1;
    r.rows = g.K;
    r.d = 1;
    r.X = g.A; r.x_dtype = g.a_dtype; r.ldx = g.sa1;
    r.b = g.B; r.b_dtype = g.b_dtype; r.sb = g.sb0;
    r.out = g.C; r.out_dtype = g.c_dtype; r.sout = 1;
    return true;
  }
  if (g.sa1 == 1 && g.K <= kRowPassMaxD && g.M * g.K >= kRowPassMinElems && g.sa0 >= g.K) {
    r.fwd = 1;
    r.rows = g.M;
    r.d = (int32_t)g.K;
    r.X = g.A; r.x_dtype = g.a_dtype; r.ldx = g.sa0;
    r.w = g.B; r.w_dtype = g.b_dtype; r.sw = g.sb0;
    r.r = g.C; r.r_dtype = g.c_dtype; r.sr = 1;
    r.e_rleaf = -1;
    return true;
  }
  if (g.sa0 == 1 && g.M <= kRowPassMaxD && g.K >= kRowPassMinRows && g.M * g.K >= kRowPassMinElems && g.sa1 >= g.M) {
    r.acc = 1;
    r.rows = g.K;
    r.d = (int32_t)g.M;
    r.X = g.A; r.x_dtype = g.a_dtype; r.ldx = g.sa1;
    r.b = g.B; r.b_dtype = g.b_dtype; r.sb = g.sb0;
    r.out = g.C; r.out_dtype = g.c_dtype; r.sout = 1;
    return true;
  }
  return false;
}

size_t gemm_scratch_bytes(const GemmArgs& g) {
  RowPassArgs r;
  return gemm_as_rowpass(g, r) ? rowpass_scratch_bytes(r) : 0;
}

int gemm_launches(const GemmArgs& g) {
  RowPassArgs r;
  return gemm_as_rowpass(g, r) ? rowpass_launches(r) : 1;
}

int launch_gemm_scratch(const GemmArgs& g, void* scratch, cudaStream_t s) {
  RowPassArgs r;
  if (gemm_as_rowpass(g, r)) {
    r.partials = (double*)scratch;
    return launch_rowpass(r, s);
  }
  return launch_gemm(g, s);
}

}  // namespace amc
