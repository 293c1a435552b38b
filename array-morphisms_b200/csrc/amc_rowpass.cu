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
#include "amc_tc.cuh"

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

// The same program with its stack in six registers (no local memory): a
// push shifts s0..s5 down, a binary operator pops one.  For programs whose
// stack stays within 6 (max_depth); leaf values come from registers by a
// select chain, so no array is indexed at run time.
__device__ __forceinline__ double leaf_sel(const double (&lv)[kMaxLeaves], int a) {
  double v = lv[0];
#pragma unroll
  for (int l = 1; l < kMaxLeaves; ++l) v = (a == l) ? lv[l] : v;
  return v;
}

// Transcendentals out of line: their code would otherwise raise the register
// count of every row pass that only does arithmetic.
__device__ __noinline__ double un_row_slow(int op, double x) {
  switch (op) {
    case AMC_OP_EXP: return exp(x);
    case AMC_OP_LOG: return log(x);
    case AMC_OP_SIN: return sin(x);
    case AMC_OP_COS: return cos(x);
    case AMC_OP_TAN: return tan(x);
    case AMC_OP_SIGMOID: return __ddiv_rn(1.0, __dadd_rn(1.0, exp(-x)));
    default: {
      double e2 = exp(__dmul_rn(2.0, x));
      return __ddiv_rn(__dsub_rn(e2, 1.0), __dadd_rn(e2, 1.0));
    }
  }
}
__device__ __noinline__ double pow_slow(double x, double y) { return pow(x, y); }

// An arithmetic program: loads, constants, conversions and the operators
// below (no transcendental).
__host__ __device__ inline bool arith_op(int op) {
  return op == AMC_OP_LOAD || op == AMC_OP_CONST || op == AMC_OP_CVT || op == AMC_OP_NEG || op == AMC_OP_ABS ||
         op == AMC_OP_FLOOR || op == AMC_OP_CEIL || op == AMC_OP_SQRT || op == AMC_OP_RELU ||
         (op >= AMC_OP_ADD && op <= AMC_OP_LE && op != AMC_OP_POW);
}

template <bool ARITH>
__device__ __forceinline__ double un_row(int op, double x) {
  switch (op) {
    case AMC_OP_NEG: return -x;
    case AMC_OP_ABS: return fabs(x);
    case AMC_OP_FLOOR: return floor(x);
    case AMC_OP_CEIL: return ceil(x);
    case AMC_OP_SQRT: return sqrt(x);
    case AMC_OP_RELU: return x > 0.0 ? x : 0.0;
    default: return ARITH ? 0.0 : un_row_slow(op, x);
  }
}

template <bool ARITH>
__device__ __forceinline__ double bin_row(int op, double x, double y) {
  switch (op) {
    case AMC_OP_ADD: return __dadd_rn(x, y);
    case AMC_OP_SUB: return __dsub_rn(x, y);
    case AMC_OP_MUL: return __dmul_rn(x, y);
    case AMC_OP_DIV: return __ddiv_rn(x, y);
    case AMC_OP_POW: return ARITH ? 0.0 : pow_slow(x, y);
    case AMC_OP_MAX: return x > y ? x : y;
    case AMC_OP_MIN: return x < y ? x : y;
    case AMC_OP_GT: return (double)(x > y);
    case AMC_OP_LT: return (double)(x < y);
    case AMC_OP_EQ: return (double)(x == y);
    case AMC_OP_GE: return (double)(x >= y);
    default: return (double)(x <= y);
  }
}

constexpr int kRegStack = 6;

template <bool ARITH>
__device__ __forceinline__ double eval_row_regs(const DProg& P, const double (&lv)[kMaxLeaves]) {
  double s0 = 0.0, s1 = 0.0, s2 = 0.0, s3 = 0.0, s4 = 0.0, s5 = 0.0;
#pragma unroll 1
  for (int pc = 0; pc < P.n; ++pc) {
    const amc_insn I = P.code[pc];
    if (I.op == AMC_OP_LOAD || I.op == AMC_OP_CONST) {
      const double v = I.op == AMC_OP_LOAD ? leaf_sel(lv, I.a) : I.imm;
      s5 = s4; s4 = s3; s3 = s2; s2 = s1; s1 = s0; s0 = v;
    } else if (I.op == AMC_OP_CVT) {
      s0 = round_to(I.a, s0);
    } else if (I.op < AMC_OP_ADD) {
      s0 = un_row<ARITH>(I.op, s0);
    } else {
      s0 = bin_row<ARITH>(I.op, s1, s0);
      s1 = s2; s2 = s3; s3 = s4; s4 = s5;
    }
  }
  return s0;
}

// Two lane-partial sums reduced across the warp in five shuffles: lanes
// 0-15 end with the sum of p0, lanes 16-31 with that of p1.
__device__ __forceinline__ double reduce2(double p0, double p1, int lane) {
  const bool hi = lane & 16;
  double b = (hi ? p1 : p0) + __shfl_xor_sync(kFull, hi ? p0 : p1, 16);
  b += __shfl_xor_sync(kFull, b, 8);
  b += __shfl_xor_sync(kFull, b, 4);
  b += __shfl_xor_sync(kFull, b, 2);
  b += __shfl_xor_sync(kFull, b, 1);
  return b;
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

// Leaf values of row i (the forward product's leaf is set by row_value).
__device__ __forceinline__ void load_row_leaves(const RowPassArgs& a, long long i, double (&lv)[kMaxLeaves]) {
#pragma unroll
  for (int l = 0; l < kMaxLeaves; ++l)
    lv[l] = (l < a.nleaf && l != a.e_rleaf) ? ld_any(a.leaf[l].ptr, a.leaf[l].dtype, i * a.leaf[l].strides[0]) : 0.0;
}

// The row value e_i: the program over the row's leaves and the forward
// product (FWD), or the stored vector b (plain transposed GEMV).
// EV: how the row program runs: 0 arithmetic on the register stack, 1 any
// program on the register stack, 2 any program on a stack in local memory
// (deeper than kRegStack), 3 the closed residual form k * (c * (p - y)).
template <bool FWD, int EV>
__device__ __forceinline__ double row_value(const RowPassArgs& a, long long i, double pr, double (&lv)[kMaxLeaves]) {
  if (FWD && EV == 3) {
    const double y = a.y_leaf < 0 ? a.y_const : leaf_sel(lv, a.y_leaf);
    double c = a.c_leaf < 0 ? a.c_const : leaf_sel(lv, a.c_leaf);
    if (a.c2_used) c = __dmul_rn(c, a.c2_leaf < 0 ? a.c2_const : leaf_sel(lv, a.c2_leaf));
    const double t = __dmul_rn(c, __dsub_rn(pr, y));
    return a.ck == 2 ? __dadd_rn(t, t) : t;
  }
  if (FWD) {
#pragma unroll
    for (int l = 0; l < kMaxLeaves; ++l) lv[l] = (l == a.e_rleaf) ? pr : lv[l];
    if constexpr (EV == 0) return eval_row_regs<true>(a.prog, lv);
    else if constexpr (EV == 1) return eval_row_regs<false>(a.prog, lv);
    else return eval_row(a.prog, lv);
  }
  return ld_any(a.b, a.b_dtype, i * a.sb);
}

// The closed residual form: the postfix program (store conversions to f64
// already dropped) parsed into a tree and matched against
//   E = ADD(X, X') with X' the same tree as X  (k = 2), or E = X (k = 1);
//   X = MUL(u, S) or MUL(S, u), u a leaf load or a constant;
//   S = SUB(LOAD rleaf, v), v a leaf load (not rleaf) or a constant.
// IEEE products and sums are commutative, and t + t = 2t exactly, so the
// closed form gives the program's values bit for bit.
struct PNode { int op, a, l, r; double imm; };

static int parse_prog(const DProg& P, std::vector<PNode>& nodes) {
  std::vector<int> st;
  for (int k = 0; k < P.n; ++k) {
    const amc_insn I = P.code[k];
    PNode n{I.op, I.a, -1, -1, I.imm};
    if (I.op == AMC_OP_LOAD || I.op == AMC_OP_CONST) {
    } else if (I.op >= AMC_OP_ADD) {
      if (st.size() < 2) return -1;
      n.r = st.back(); st.pop_back();
      n.l = st.back(); st.pop_back();
    } else {
      return -1;   // unary operators and stores do not occur in the form
    }
    nodes.push_back(n);
    st.push_back((int)nodes.size() - 1);
  }
  return st.size() == 1 ? st[0] : -1;
}

static bool same_tree(const std::vector<PNode>& t, int x, int y) {
  const PNode &a = t[x], &b = t[y];
  if (a.op != b.op) return false;
  if (a.op == AMC_OP_LOAD) return a.a == b.a;
  if (a.op == AMC_OP_CONST) return a.imm == b.imm;
  return same_tree(t, a.l, b.l) && same_tree(t, a.r, b.r);
}

static bool leaf_or_const(const PNode& n, int* leaf, double* c) {
  if (n.op == AMC_OP_LOAD) { *leaf = n.a; return true; }
  if (n.op == AMC_OP_CONST) { *leaf = -1; *c = n.imm; return true; }
  return false;
}

void match_closed_form(RowPassArgs& a) {
  a.closed = 0;
  if (!a.fwd || !a.acc || !a.prog.all_float) return;
  std::vector<PNode> t;
  int root = parse_prog(a.prog, t);
  if (root < 0) return;
  int x = root, k = 1;
  if (t[root].op == AMC_OP_ADD && same_tree(t, t[root].l, t[root].r)) { x = t[root].l; k = 2; }
  if (t[x].op != AMC_OP_MUL) return;
  int sidx = -1, uidx = -1;
  if (t[t[x].r].op == AMC_OP_SUB) { sidx = t[x].r; uidx = t[x].l; }
  else if (t[t[x].l].op == AMC_OP_SUB) { sidx = t[x].l; uidx = t[x].r; }
  else return;
  const PNode& S = t[sidx];
  if (t[S.l].op != AMC_OP_LOAD || t[S.l].a != a.e_rleaf) return;
  int cl = -1, c2l = -1, yl = -1, c2u = 0;
  double cc = 0.0, c2c = 0.0, yc = 0.0;
  const PNode& U = t[uidx];
  if (U.op == AMC_OP_MUL) {   // a coefficient that is itself a product of two leaves or constants
    if (!leaf_or_const(t[U.l], &cl, &cc) || !leaf_or_const(t[U.r], &c2l, &c2c)) return;
    c2u = 1;
  } else if (!leaf_or_const(U, &cl, &cc)) {
    return;
  }
  if (cl == a.e_rleaf || (c2u && c2l == a.e_rleaf)) return;
  if (!leaf_or_const(t[S.r], &yl, &yc) || yl == a.e_rleaf) return;
  a.closed = 1;
  a.ck = k;
  a.c_leaf = cl; a.c_const = cc;
  a.c2_used = c2u; a.c2_leaf = c2l; a.c2_const = c2c;
  a.y_leaf = yl; a.y_const = yc;
}

int row_eval_mode(const RowPassArgs& a) {
  const DProg& P = a.prog;
  if (a.closed) return 3;
  if (P.max_depth > kRegStack) return 2;
  for (int k = 0; k < P.n; ++k)
    if (!arith_op(P.code[k].op)) return 1;
  return 0;
}

// G = 4 rows per group; after the group's reduction lane q * (32 / G) owns
// row q.  The single products run here; the GEMV pair (FWD and ACC) runs in
// k_gemv_pair_tma, k_gemv_pair or, for other widths, k_rowpass_any.
template <typename T, int KPL, bool FWD, bool ACC, int G, int EV>
__global__ void __launch_bounds__(kRowBlock) k_rowpass(const __grid_constant__ RowPassArgs a) {
  constexpr int D = 32 * KPL;
  constexpr int LPR = 32 / G;   // lanes per owned row after the reduction
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
  const int q_own = lane / LPR;
  const bool owner = (lane % LPR) == 0;
  long long i = r0;
  for (; i + G <= r1; i += G) {
    double x[G][KPL];
#pragma unroll
    for (int q = 0; q < G; ++q) {
      const T* px = X + (i + q) * a.ldx + lane;
#pragma unroll
      for (int j = 0; j < KPL; ++j) x[q][j] = ld_stream(px + 32 * j);
    }
    double lv[kMaxLeaves];
    if (ACC && FWD && owner) load_row_leaves(a, i + q_own, lv);
    double ev = 0.0;
    if (FWD) {
      double p[G];
#pragma unroll
      for (int q = 0; q < G; ++q) {
        p[q] = 0.0;
#pragma unroll
        for (int j = 0; j < KPL; ++j) p[q] = fma(x[q][j], wv[j], p[q]);
      }
      static_assert(G == 4, "the single products run 4 rows per group");
      const double s = reduce4(p[0], p[1], p[2], p[3], lane);
      if (owner) {
        const double pr = fwd_store(a, i + q_own, s);
        if (ACC) ev = row_value<true, EV>(a, i + q_own, pr, lv);
      }
    } else if (owner) {
      ev = row_value<false, EV>(a, i + q_own, 0.0, lv);
    }
    if (ACC) {
#pragma unroll
      for (int q = 0; q < G; ++q) {
        const double e = __shfl_sync(kFull, ev, LPR * q);
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
        if (ACC) ev = row_value<true, EV>(a, i, pr, lv);
      }
    } else if (lane == 0) {
      ev = row_value<false, EV>(a, i, 0.0, lv);
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

// The GEMV pair for d = 32 * NW: NW warps, warp w owning columns
// [32w, 32w + 32), 32 rows per iteration.  Each lane holds its column of the
// 32 rows in registers; the warp's partial dot products of the 32 rows are
// transposed across the lanes by a halving shuffle reduction (lane r ends
// with row r's partial), the NW partials are added in warp order by warp 0,
// whose lane r then stores p_r and runs the row program for row r (one
// program evaluation serves 32 rows); every lane then accumulates its column
// of X^T e from the rows still in its registers.  X is read once.
template <typename T, int NW, int EV>
__global__ void __launch_bounds__(32 * NW, 16 / NW) k_gemv_pair(const __grid_constant__ RowPassArgs a) {
  __shared__ double part[NW][32];
  __shared__ double e_sm[32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int col = 32 * warp + lane;
  const double wv = ld_any(a.w, a.w_dtype, (long long)col * a.sw);
  const long long rb = a.rows * blockIdx.x / gridDim.x, re = a.rows * (blockIdx.x + 1) / gridDim.x;
  const T* X = (const T*)a.X + col;
  double acc0 = 0.0, acc1 = 0.0;
  for (long long i0 = rb; i0 < re; i0 += 32) {
    const int nr = (int)((re - i0) < 32 ? (re - i0) : 32);
    double x[32];
#pragma unroll
    for (int r = 0; r < 32; ++r) x[r] = r < nr ? ld_stream(X + (i0 + r) * a.ldx) : 0.0;
    double lv[kMaxLeaves];
    if (warp == 0 && lane < nr) load_row_leaves(a, i0 + lane, lv);
    // halving reduction of the 32 partial products: lane r ends with row r's
    double t16[16], t8[8], t4[4], t2[2];
    {
      const bool h = lane & 16;
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const double lo = x[j] * wv, hi = x[16 + j] * wv;
        t16[j] = (h ? hi : lo) + __shfl_xor_sync(kFull, h ? lo : hi, 16);
      }
    }
    {
      const bool h = lane & 8;
#pragma unroll
      for (int j = 0; j < 8; ++j) t8[j] = (h ? t16[8 + j] : t16[j]) + __shfl_xor_sync(kFull, h ? t16[j] : t16[8 + j], 8);
    }
    {
      const bool h = lane & 4;
#pragma unroll
      for (int j = 0; j < 4; ++j) t4[j] = (h ? t8[4 + j] : t8[j]) + __shfl_xor_sync(kFull, h ? t8[j] : t8[4 + j], 4);
    }
    {
      const bool h = lane & 2;
#pragma unroll
      for (int j = 0; j < 2; ++j) t2[j] = (h ? t4[2 + j] : t4[j]) + __shfl_xor_sync(kFull, h ? t4[j] : t4[2 + j], 2);
    }
    const bool h1 = lane & 1;
    const double mine = (h1 ? t2[1] : t2[0]) + __shfl_xor_sync(kFull, h1 ? t2[0] : t2[1], 1);
    if (NW > 1) part[warp][lane] = mine;
    if (NW > 1) __syncthreads();
    if (warp == 0) {
      double pv = mine;
      if (NW > 1) {
        pv = part[0][lane];
#pragma unroll
        for (int w = 1; w < NW; ++w) pv += part[w][lane];
      }
      double ev = 0.0;
      if (lane < nr) {
        const double pr = fwd_store(a, i0 + lane, pv);
        ev = row_value<true, EV>(a, i0 + lane, pr, lv);
      }
      e_sm[lane] = ev;
    }
    __syncthreads();
#pragma unroll
    for (int r = 0; r < 32; r += 2) {
      acc0 = fma(x[r], e_sm[r], acc0);
      acc1 = fma(x[r + 1], e_sm[r + 1], acc1);
    }
    __syncthreads();   // e_sm and part are rewritten next iteration
  }
  a.partials[(long long)blockIdx.x * (32 * NW) + col] = acc0 + acc1;
}

// The GEMV pair as a TMA-fed pipeline, for contiguous rows (ldx == d,
// d = 32 * KPL).  One CTA per SM:
//   producer warp   streams 32-row tiles of X (32 * d elements, contiguous)
//                   into NS shared-memory stages with cp.async.bulk (no
//                   multicast), completion counted on full[stage];
//   8 compute warps  warp w takes rows 4w..4w+3 of each tile, lanes over the
//                   columns (lane + 32 j): p of its 4 rows by a fixed shuffle
//                   reduction; lanes 0, 8, 16, 24 store p_r and run the row
//                   program for their row (its leaves fetched one tile
//                   ahead); e_r goes back to every lane by a shuffle, and the
//                   4 rows, still in registers, accumulate X^T e into the
//                   warp's column accumulators.  The stage is released as soon
//                   as every warp has its rows, so the producer keeps the other
//                   stages in flight.
// No warp waits on another warp's arithmetic: a tile costs each warp one
// dependent chain (reduction, program, shuffle), and the 8 warps run theirs
// side by side.  At the end the 8 warps' accumulators are added in warp
// order.  Every wait is bounded: on expiry the waiting role records
// AMC_ERR_TIMEOUT, raises the CTA's abort flag and leaves; the producer waits
// (bounded) for its copies in flight before returning.
__device__ int g_rowpass_error;

constexpr int kPairWaitLimit = 1 << 22;
constexpr int kPairCompute = 8;     // compute warps
constexpr int kPairRows = 32;       // rows per tile
constexpr int kPairRpw = kPairRows / kPairCompute;   // rows per compute warp per tile
constexpr int kPairThreads = 32 * (kPairCompute + 1);
constexpr int kPairChunks = 4;      // bulk copies per tile (8 rows each), each warp waits for its own
static_assert(kPairRows % kPairChunks == 0 && (kPairRows / kPairChunks) % kPairRpw == 0, "a warp's rows lie in one chunk");

template <typename T, int KPL, int EV>
__global__ void __launch_bounds__(kPairThreads, 1) k_gemv_pair_tma(const __grid_constant__ RowPassArgs a, int ns) {
  extern __shared__ __align__(128) unsigned char pair_sm[];
  constexpr int D = 32 * KPL;
  constexpr int TILE = kPairRows * D;           // elements per stage
  constexpr int NCH = kPairChunks;               // copies per stage, one barrier each
  constexpr int CROWS = kPairRows / NCH;
  T* xs = (T*)pair_sm;
  uint64_t* full = (uint64_t*)(pair_sm + (size_t)ns * TILE * sizeof(T));   // [ns][NCH]
  uint64_t* empty = full + ns * NCH;
  volatile int* abort_flag = (volatile int*)(empty + ns);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const long long rb = a.rows * blockIdx.x / gridDim.x, re = a.rows * (blockIdx.x + 1) / gridDim.x;
  const long long nt = (re - rb + kPairRows - 1) / kPairRows;   // tiles of this CTA
  if (threadIdx.x == 0) {
    for (int k = 0; k < ns; ++k) {
      for (int c = 0; c < NCH; ++c) tc::mbar_init(&full[k * NCH + c], 1);
      tc::mbar_init(&empty[k], kPairCompute);
    }
    *abort_flag = 0;
    tc::mbar_fence_init();
  }
  __syncthreads();
  auto fail_wait = [&]() {
    atomicExch(&g_rowpass_error, AMC_ERR_TIMEOUT);
    *abort_flag = 1;
  };
  auto rows_of = [&](long long s) -> int {
    const long long left = re - rb - (long long)kPairRows * s;
    return (int)(left < kPairRows ? left : kPairRows);
  };
  const T* Xg = (const T*)a.X;
  if (warp == kPairCompute) {
    // ---------------------------------------------------------------- producer
    if (lane != 0) return;
    const uint64_t policy = tc::l2_policy_evict_first();   // X is read once
    long long issued = 0;
    for (long long s = 0; s < nt && !*abort_flag; ++s) {
      const int st = (int)(s % ns);
      if (s >= ns && !tc::mbar_wait(&empty[st], (uint32_t)(((s - ns) / ns) & 1), kPairWaitLimit)) {
        fail_wait();
        break;
      }
      const int nr = rows_of(s);
      const T* src = Xg + (rb + (long long)kPairRows * s) * D;
      for (int c = 0; c < NCH; ++c) {
        const int cr = nr - c * CROWS < CROWS ? nr - c * CROWS : CROWS;
        uint64_t* bar = &full[st * NCH + c];
        if (cr <= 0) {
          tc::mbar_arrive(bar);   // an empty chunk of the last tile completes at once
          continue;
        }
        const uint32_t bytes = (uint32_t)((long long)cr * D * sizeof(T));
        tc::mbar_expect_tx(bar, bytes);
        tc::bulk_load_1d_hint(xs + (size_t)st * TILE + (size_t)c * CROWS * D, src + (size_t)c * CROWS * D, bytes, bar,
                              policy);
      }
      ++issued;
    }
    // copies still in flight complete before the CTA's shared memory goes away
    for (long long s = issued > ns ? issued - ns : 0; s < issued; ++s)
      for (int c = 0; c < NCH; ++c)
        if (!tc::mbar_wait(&full[(s % ns) * NCH + c], (uint32_t)((s / ns) & 1), kPairWaitLimit)) fail_wait();
    return;
  }
  // ---------------------------------------------------------------- compute warps
  double wv[KPL], acc[KPL];
#pragma unroll
  for (int j = 0; j < KPL; ++j) {
    wv[j] = ld_any(a.w, a.w_dtype, (long long)(lane + 32 * j) * a.sw);
    acc[j] = 0.0;
  }
  static_assert(kPairRpw == 4, "four rows per compute warp");
  const int row0 = kPairRpw * warp;            // the warp's first row within a tile
  const int q_own = lane >> 3;                   // after reduce4, lane 8q holds row q's p
  const bool owner = (lane & 7) == 0;
  double lv[kMaxLeaves];
  if (owner && nt > 0 && row0 + q_own < rows_of(0)) load_row_leaves(a, rb + row0 + q_own, lv);
  double rsum = 0.0;    // the row sum of this owner lane's rows, in row order
  bool ok = true;
  for (long long s = 0; s < nt && !*abort_flag; ++s) {
    const int st = (int)(s % ns);
    if (!tc::mbar_wait(&full[st * NCH + row0 / CROWS], (uint32_t)((s / ns) & 1), kPairWaitLimit)) {
      ok = false;
      break;
    }
    const int nr = rows_of(s);
    const T* xt = xs + (size_t)st * TILE + (size_t)row0 * D + lane;
    double x[kPairRpw][KPL];
#pragma unroll
    for (int q = 0; q < kPairRpw; ++q)
#pragma unroll
      for (int j = 0; j < KPL; ++j) x[q][j] = row0 + q < nr ? (double)xt[q * D + 32 * j] : 0.0;
    // the rows are in registers: the stage goes back to the producer
    __syncwarp();
    if (lane == 0) tc::mbar_arrive(&empty[st]);
    double p[kPairRpw];
#pragma unroll
    for (int q = 0; q < kPairRpw; ++q) {
      p[q] = 0.0;
#pragma unroll
      for (int j = 0; j < KPL; ++j) p[q] = fma(x[q][j], wv[j], p[q]);
    }
    const double sum = reduce4(p[0], p[1], p[2], p[3], lane);
    double ev = 0.0;
    const long long r = rb + (long long)kPairRows * s + row0 + q_own;
    if (owner && row0 + q_own < nr) {
      const double pr = fwd_store(a, r, sum);
      ev = row_value<true, EV>(a, r, pr, lv);
      if (EV == 3 && a.rsum) {
        const double t = __dsub_rn(pr, a.rsum_y_leaf < 0 ? a.rsum_y_const : leaf_sel(lv, a.rsum_y_leaf));
        rsum = __dadd_rn(rsum, __dmul_rn(t, t));
      }
    }
    // the next tile's leaves, while this tile's rows accumulate
    if (owner && s + 1 < nt && row0 + q_own < rows_of(s + 1)) load_row_leaves(a, r + kPairRows, lv);
#pragma unroll
    for (int q = 0; q < kPairRpw; ++q) {
      const double e = __shfl_sync(kFull, ev, 8 * q);
#pragma unroll
      for (int j = 0; j < KPL; ++j) acc[j] = fma(x[q][j], e, acc[j]);
    }
  }
  if (!ok) fail_wait();
  // the warps' accumulators added in warp order (through the stage memory,
  // which no copy targets any more once every compute warp is here: each
  // warp waited for every tile's copy)
  asm volatile("bar.sync 1, %0;" ::"r"(kPairCompute * 32) : "memory");
  if (!*abort_flag) {
    double* red = (double*)pair_sm;   // [kPairCompute][D], then [kPairCompute] row sums
#pragma unroll
    for (int j = 0; j < KPL; ++j) red[warp * D + lane + 32 * j] = acc[j];
    if (EV == 3 && a.rsum) {
      // the 4 owner lanes' sums in row order (lanes 0, 8, 16, 24), then the warps in order
      const double r8 = __shfl_sync(kFull, rsum, 8), r16 = __shfl_sync(kFull, rsum, 16),
                   r24 = __shfl_sync(kFull, rsum, 24);
      if (lane == 0) red[kPairCompute * D + warp] = ((rsum + r8) + r16) + r24;
    }
    asm volatile("bar.sync 1, %0;" ::"r"(kPairCompute * 32) : "memory");
    for (int k = threadIdx.x; k < D; k += kPairCompute * 32) {
      double t = red[k];
#pragma unroll
      for (int w = 1; w < kPairCompute; ++w) t += red[w * D + k];
      a.partials[(long long)blockIdx.x * D + k] = t;
    }
    if (EV == 3 && a.rsum && threadIdx.x == 0) {
      double t = red[kPairCompute * D];
#pragma unroll
      for (int w = 1; w < kPairCompute; ++w) t += red[kPairCompute * D + w];
      a.partials[(long long)gridDim.x * D + blockIdx.x] = t;
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
        if (ACC) ev = row_value<true, 2>(a, i, pr, lv);
      }
    } else if (lane == 0) {
      ev = row_value<false, 2>(a, i, 0.0, lv);
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
  // four independent chains, so eight loads per thread are in flight at
  // once; their fixed combination keeps the result deterministic
  double s0 = 0.0, s1 = 0.0, s2 = 0.0, s3 = 0.0;
  long long k = b0 + threadIdx.x;
  for (; k + 3 * kRowBlock < b1; k += 4 * kRowBlock) {
    const double x0 = (double)__ldcs(x + k * sx), y0 = (double)__ldcs(y + k * sy);
    const double x1 = (double)__ldcs(x + (k + kRowBlock) * sx), y1 = (double)__ldcs(y + (k + kRowBlock) * sy);
    const double x2 = (double)__ldcs(x + (k + 2 * kRowBlock) * sx), y2 = (double)__ldcs(y + (k + 2 * kRowBlock) * sy);
    const double x3 = (double)__ldcs(x + (k + 3 * kRowBlock) * sx), y3 = (double)__ldcs(y + (k + 3 * kRowBlock) * sy);
    s0 = fma(x0, y0, s0);
    s1 = fma(x1, y1, s1);
    s2 = fma(x2, y2, s2);
    s3 = fma(x3, y3, s3);
  }
  for (; k < b1; k += kRowBlock) s0 = fma((double)__ldcs(x + k * sx), (double)__ldcs(y + k * sy), s0);
  double s = (s0 + s1) + (s2 + s3);
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
                                                        int out_dtype, long long sout, double alpha, double beta,
                                                        double div = 0.0) {
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
    if (div != 0.0) v = __ddiv_rn(v, div);
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

template <typename T, bool FWD, bool ACC, int EV, int G>
int launch_kpl(const RowPassArgs& a, int grid, cudaStream_t s) {
  switch (a.d) {
    case 32: k_rowpass<T, 1, FWD, ACC, G, EV><<<grid, kRowBlock, 0, s>>>(a); return AMC_OK;
    case 64: k_rowpass<T, 2, FWD, ACC, G, EV><<<grid, kRowBlock, 0, s>>>(a); return AMC_OK;
    case 128: k_rowpass<T, 4, FWD, ACC, G, EV><<<grid, kRowBlock, 0, s>>>(a); return AMC_OK;
    case 256: k_rowpass<T, 8, FWD, ACC, G, EV><<<grid, kRowBlock, 0, s>>>(a); return AMC_OK;
    default: return launch_any<T, FWD, ACC>(a, grid, s);
  }
}

std::atomic<uint64_t> g_pair_smem_done[2][4][4];

template <typename T, int KPL, int EV>
int launch_pair_tma(const RowPassArgs& a, int grid, cudaStream_t s) {
  const int stage = kPairRows * 32 * KPL * (int)sizeof(T);
  int ns = (200 * 1024) / stage;
  ns = ns > 8 ? 8 : ns;
  // the stages also hold the final warp reduction (kPairCompute x d doubles),
  // which is at most a quarter of the 8 stages a 32-column f32 tile gets
  const size_t stages = (size_t)ns * stage;
  static_assert(kPairCompute * 33 * sizeof(double) <= 8 * kPairRows * 32 * sizeof(float), "reduction fits the stages");
  const size_t smem = stages + (kPairChunks + 1) * ns * 8 + 16;
  const int ki = KPL == 1 ? 0 : KPL == 2 ? 1 : KPL == 4 ? 2 : 3;
  int rc = smem_attr_once(k_gemv_pair_tma<T, KPL, EV>, (int)smem, g_pair_smem_done[sizeof(T) == 8][ki][EV]);
  if (rc) return rc;
  k_gemv_pair_tma<T, KPL, EV><<<grid, kPairThreads, smem, s>>>(a, ns);
  return AMC_OK;
}

// The GEMV pair runs the TMA pipeline (one CTA per SM) on contiguous rows
// whose tiles start on 16-byte boundaries.
bool pair_tma_ok(const RowPassArgs& a) {
  return a.fwd && a.acc && a.ldx == a.d && ((uintptr_t)a.X & 15) == 0 &&
         (a.d == 32 || a.d == 64 || a.d == 128 || a.d == 256);
}

template <typename T, int EV>
int launch_pair(const RowPassArgs& a, int grid, cudaStream_t s) {
  if (pair_tma_ok(a)) {
    switch (a.d) {
      case 32: return launch_pair_tma<T, 1, EV>(a, grid, s);
      case 64: return launch_pair_tma<T, 2, EV>(a, grid, s);
      case 128: return launch_pair_tma<T, 4, EV>(a, grid, s);
      case 256: return launch_pair_tma<T, 8, EV>(a, grid, s);
      default: break;
    }
  }
  switch (a.d) {
    case 32: k_gemv_pair<T, 1, EV><<<grid, 32, 0, s>>>(a); return AMC_OK;
    case 64: k_gemv_pair<T, 2, EV><<<grid, 64, 0, s>>>(a); return AMC_OK;
    case 128: k_gemv_pair<T, 4, EV><<<grid, 128, 0, s>>>(a); return AMC_OK;
    case 256: k_gemv_pair<T, 8, EV><<<grid, 256, 0, s>>>(a); return AMC_OK;
    default: return launch_any<T, true, true>(a, grid, s);
  }
}

template <typename T, bool FWD, bool ACC>
int launch_mode(const RowPassArgs& a, int grid, cudaStream_t s) {
  if (!(FWD && ACC)) return launch_kpl<T, FWD, ACC, 0, 4>(a, grid, s);
  switch (row_eval_mode(a)) {
    case 0: return launch_pair<T, 0>(a, grid, s);
    case 1: return launch_pair<T, 1>(a, grid, s);
    case 3: return launch_pair<T, 3>(a, grid, s);
    default: return launch_pair<T, 2>(a, grid, s);
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

void rowpass_prepare(RowPassArgs& a) { match_closed_form(a); }

int rowpass_check_error() {
  int e = 0;
  AMC_CUDA(cudaMemcpyFromSymbol(&e, g_rowpass_error, sizeof(int)));
  if (e) {
    int z = 0;
    AMC_CUDA(cudaMemcpyToSymbol(g_rowpass_error, &z, sizeof(int)));
    return fail(e, "row pass: a bounded wait of the GEMV-pair pipeline gave up");
  }
  return AMC_OK;
}

int rowpass_grid(int64_t rows) {
  long long g = (long long)num_sms() * 4;
  long long need = (rows + 31) / 32;   // at least 32 rows per CTA
  if (need < g) g = need;
  return (int)(g < 1 ? 1 : g);
}

size_t rowpass_scratch_bytes(const RowPassArgs& a) {
  if (a.dot) return (size_t)rowpass_grid(a.rows) * sizeof(double);
  if (!a.acc) return 0;
  // the GEMV pair also keeps one row-sum partial per CTA after the d columns
  return (size_t)rowpass_grid(a.rows) * (size_t)(a.d + (a.fwd ? 1 : 0)) * sizeof(double);
}

bool rowpass_pair_tma(const RowPassArgs& a) { return pair_tma_ok(a); }

int rowpass_ctas(const RowPassArgs& a) {
  int grid = rowpass_grid(a.rows);
  if (pair_tma_ok(a) && grid > num_sms()) grid = num_sms();
  return grid;
}

int launch_rowsum_finish(const double* partials, int n, void* out, int out_dtype, double div, cudaStream_t s) {
  k_rowpass_reduce<<<1, 256, 0, s>>>(partials, n, 1, out, out_dtype, 1, 1.0, 0.0, div);
  AMC_CUDA(cudaGetLastError());
  return AMC_OK;
}

int launch_rowpass(const RowPassArgs& a, cudaStream_t s) {
  if (a.rows < 0 || a.d < 1 || a.d > kRowPassMaxD || (!a.fwd && !a.acc && !a.dot))
    return fail(AMC_ERR_INVALID, "row pass: bad shape");
  if ((a.acc || a.dot) && !a.partials) return fail(AMC_ERR_INVALID, "row pass: no scratch for the partial sums");
  if (a.fwd && a.acc && (a.e_rleaf < 0 || a.e_rleaf >= a.nleaf || a.nleaf > kMaxLeaves))
    return fail(AMC_ERR_INVALID, "row pass: the row program does not read the forward product");
  if (fault_injected("launch")) return fail(AMC_ERR_INJECTED, "row pass: injected launch failure (AMC_FAULT=launch)");
  // the CTAs that write partial rows (the reduce adds exactly these)
  const int grid = rowpass_ctas(a);
  if (a.rsum && !(a.closed && pair_tma_ok(a)))
    return fail(AMC_ERR_INVALID, "row pass: a row sum needs the closed row form on contiguous rows");
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
