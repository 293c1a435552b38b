// Generic device kernels of the realization engine:
//   - fused element-wise programs over strided views   (realization.scm:876-997)
//   - ordered reductions                                (realization.scm:1309-1388)
//   - pad / im2col / col2im / stack-concat gathers      (realization.scm:1003-1268, 1425-1459)
//   - double-accumulating GEMM                          (blas-exec.scm:405-458)
//   - reference-order streaming attention               (realization.scm:279-396)
// Numeric semantics follow the reference's Scheme numbers: inexact values are
// IEEE doubles, exact values are 64-bit integers, and a node's result is
// converted only when stored (typed-vector-set!, core.scm:649-658).
#include <cfloat>
#include <cmath>

#include "amc_internal.h"

namespace amc {

// ------------------------------------------------------------------ numbers
struct Num {
  double f;
  long long i;
  int exact;
};

__device__ __forceinline__ Num nfl(double f) { Num r; r.f = f; r.i = 0; r.exact = 0; return r; }
__device__ __forceinline__ Num nex(long long i) { Num r; r.f = (double)i; r.i = i; r.exact = 1; return r; }
__device__ __forceinline__ double as_f(const Num& a) { return a.exact ? (double)a.i : a.f; }
__device__ __forceinline__ bool dtype_is_float_d(int d) { return d == AMC_F32 || d == AMC_F64; }

__device__ __forceinline__ Num load_num(const void* p, int dtype, long long k) {
  switch (dtype) {
    case AMC_F32: return nfl((double)__ldg((const float*)p + k));
    case AMC_F64: return nfl(__ldg((const double*)p + k));
    case AMC_S32: return nex(__ldg((const int*)p + k));
    case AMC_S64: return nex(__ldg((const long long*)p + k));
    case AMC_U32: return nex((long long)__ldg((const unsigned*)p + k));
    default: return nex((long long)__ldg((const unsigned long long*)p + k));
  }
}

__device__ __forceinline__ double load_f(const void* p, int dtype, long long k) {
  return dtype == AMC_F32 ? (double)__ldg((const float*)p + k) : __ldg((const double*)p + k);
}

__device__ __forceinline__ long long trunc_i(const Num& x) { return x.exact ? x.i : (long long)trunc(x.f); }

__device__ __forceinline__ Num round_store(int dtype, const Num& x) {
  switch (dtype) {
    case AMC_F32: return nfl((double)__double2float_rn(as_f(x)));
    case AMC_F64: return nfl(as_f(x));
    case AMC_S32: return nex((int)trunc_i(x));
    case AMC_S64: return nex(trunc_i(x));
    case AMC_U32: { long long t = trunc_i(x); return nex((unsigned)(t < 0 ? -t : t)); }
    default: { long long t = trunc_i(x); return nex(t < 0 ? -t : t); }
  }
}

__device__ __forceinline__ void store_num(void* p, int dtype, long long k, const Num& x) {
  switch (dtype) {
    case AMC_F32: ((float*)p)[k] = __double2float_rn(as_f(x)); break;
    case AMC_F64: ((double*)p)[k] = as_f(x); break;
    case AMC_S32: ((int*)p)[k] = (int)trunc_i(x); break;
    case AMC_S64: ((long long*)p)[k] = trunc_i(x); break;
    case AMC_U32: { long long t = trunc_i(x); ((unsigned*)p)[k] = (unsigned)(t < 0 ? -t : t); } break;
    default: { long long t = trunc_i(x); ((unsigned long long*)p)[k] = (unsigned long long)(t < 0 ? -t : t); } break;
  }
}

__device__ __forceinline__ long long ipow_d(long long a, long long b) {
  long long r = 1;
  while (b > 0) { if (b & 1) r *= a; a *= a; b >>= 1; }
  return r;
}

__device__ __forceinline__ Num un_op(int op, const Num& a) {
  double x = as_f(a);
  switch (op) {
    case AMC_OP_NEG: return a.exact ? nex(-a.i) : nfl(-a.f);
    case AMC_OP_ABS: return a.exact ? nex(a.i < 0 ? -a.i : a.i) : nfl(fabs(a.f));
    case AMC_OP_FLOOR: return a.exact ? a : nfl(floor(a.f));
    case AMC_OP_CEIL: return a.exact ? a : nfl(ceil(a.f));
    case AMC_OP_SQRT:
      if (a.exact && a.i >= 0) {
        long long r = llround(sqrt((double)a.i));
        if (r * r == a.i) return nex(r);
      }
      return nfl(sqrt(x));
    case AMC_OP_EXP: return nfl(exp(x));
    case AMC_OP_LOG: return nfl(log(x));
    case AMC_OP_SIN: return nfl(sin(x));
    case AMC_OP_COS: return nfl(cos(x));
    case AMC_OP_TAN: return nfl(tan(x));
    case AMC_OP_RELU: return nfl(x > 0.0 ? x : 0.0);
    case AMC_OP_SIGMOID: return nfl(__ddiv_rn(1.0, __dadd_rn(1.0, exp(-x))));
    case AMC_OP_TANH: { double e2 = exp(__dmul_rn(2.0, x)); return nfl(__ddiv_rn(__dsub_rn(e2, 1.0), __dadd_rn(e2, 1.0))); }
  }
  return nfl(NAN);
}

__device__ __forceinline__ Num bin_op(int op, const Num& a, const Num& b) {
  bool ex = a.exact && b.exact;
  double x = as_f(a), y = as_f(b);
  switch (op) {
    case AMC_OP_ADD: return ex ? nex(a.i + b.i) : nfl(__dadd_rn(x, y));
    case AMC_OP_SUB: return ex ? nex(a.i - b.i) : nfl(__dsub_rn(x, y));
    case AMC_OP_MUL: return ex ? nex(a.i * b.i) : nfl(__dmul_rn(x, y));
    case AMC_OP_DIV:
      if (ex) {
        if (b.i != 0 && a.i % b.i == 0) return nex(a.i / b.i);
        return nfl(__ddiv_rn((double)a.i, (double)b.i));
      }
      return nfl(__ddiv_rn(x, y));
    case AMC_OP_POW: return (ex && b.i >= 0) ? nex(ipow_d(a.i, b.i)) : nfl(pow(x, y));
    case AMC_OP_MAX: return ex ? nex(a.i > b.i ? a.i : b.i) : nfl(x > y ? x : y);
    case AMC_OP_MIN: return ex ? nex(a.i < b.i ? a.i : b.i) : nfl(x < y ? x : y);
    case AMC_OP_GT: return nfl(ex ? (double)(a.i > b.i) : (double)(x > y));
    case AMC_OP_LT: return nfl(ex ? (double)(a.i < b.i) : (double)(x < y));
    case AMC_OP_EQ: return nfl(ex ? (double)(a.i == b.i) : (double)(x == y));
    case AMC_OP_GE: return nfl(ex ? (double)(a.i >= b.i) : (double)(x >= y));
    case AMC_OP_LE: return nfl(ex ? (double)(a.i <= b.i) : (double)(x <= y));
  }
  return nfl(NAN);
}

// Tagged evaluation (exact integers and doubles).  With OV, leaf `ov` is not
// read from memory: its loads yield `ovv` (a GEMM epilogue's own product, a
// scan's running accumulator).
template <bool OV = false>
__device__ Num eval_prog(const DProg& P, const DLeaf* L, const long long* off, int ov = -1, Num ovv = Num()) {
  Num st[AMC_STACK_MAX];
  int sp = 0;
  for (int pc = 0; pc < P.n; ++pc) {
    const amc_insn I = P.code[pc];
    switch (I.op) {
      case AMC_OP_LOAD:
        st[sp++] = (OV && I.a == ov) ? ovv : load_num(L[I.a].ptr, L[I.a].dtype, off[I.a]);
        break;
      case AMC_OP_CONST: st[sp++] = nfl(I.imm); break;
      case AMC_OP_ICONST: st[sp++] = nex((long long)I.imm); break;
      case AMC_OP_CVT: st[sp - 1] = round_store(I.a, st[sp - 1]); break;
      default:
        if (I.op < AMC_OP_ADD) st[sp - 1] = un_op(I.op, st[sp - 1]);
        else { st[sp - 2] = bin_op(I.op, st[sp - 2], st[sp - 1]); --sp; }
    }
  }
  return st[0];
}

// Inexact-only evaluation: every value is a double.
__device__ __forceinline__ double un_f(int op, double x) {
  switch (op) {
    case AMC_OP_NEG: return -x;
    case AMC_OP_ABS: return fabs(x);
    case AMC_OP_FLOOR: return floor(x);
    case AMC_OP_CEIL: return ceil(x);
    case AMC_OP_SQRT: return sqrt(x);
    case AMC_OP_EXP: return exp(x);
    case AMC_OP_LOG: return log(x);
    case AMC_OP_SIN: return sin(x);
    case AMC_OP_COS: return cos(x);
    case AMC_OP_TAN: return tan(x);
    case AMC_OP_RELU: return x > 0.0 ? x : 0.0;
    case AMC_OP_SIGMOID: return __ddiv_rn(1.0, __dadd_rn(1.0, exp(-x)));
    case AMC_OP_TANH: { double e2 = exp(__dmul_rn(2.0, x)); return __ddiv_rn(__dsub_rn(e2, 1.0), __dadd_rn(e2, 1.0)); }
  }
  return NAN;
}

__device__ __forceinline__ double bin_f(int op, double x, double y) {
  switch (op) {
    case AMC_OP_ADD: return __dadd_rn(x, y);
    case AMC_OP_SUB: return __dsub_rn(x, y);
    case AMC_OP_MUL: return __dmul_rn(x, y);
    case AMC_OP_DIV: return __ddiv_rn(x, y);
    case AMC_OP_POW: return pow(x, y);
    case AMC_OP_MAX: return x > y ? x : y;
    case AMC_OP_MIN: return x < y ? x : y;
    case AMC_OP_GT: return (double)(x > y);
    case AMC_OP_LT: return (double)(x < y);
    case AMC_OP_EQ: return (double)(x == y);
    case AMC_OP_GE: return (double)(x >= y);
    case AMC_OP_LE: return (double)(x <= y);
  }
  return NAN;
}

__device__ __forceinline__ double round_f(int dtype, double x) {
  switch (dtype) {
    case AMC_F32: return (double)__double2float_rn(x);
    case AMC_F64: return x;
    case AMC_S32: return (double)(int)(long long)trunc(x);
    case AMC_S64: return (double)(long long)trunc(x);
    case AMC_U32: { long long t = (long long)trunc(x); return (double)(unsigned)(t < 0 ? -t : t); }
    default: { long long t = (long long)trunc(x); return (double)(t < 0 ? -t : t); }
  }
}

template <bool OV = false>
__device__ double eval_prog_f(const DProg& P, const DLeaf* L, const long long* off, int ov = -1, double ovv = 0.0) {
  double st[AMC_STACK_MAX];
  int sp = 0;
  for (int pc = 0; pc < P.n; ++pc) {
    const amc_insn I = P.code[pc];
    switch (I.op) {
      case AMC_OP_LOAD: st[sp++] = (OV && I.a == ov) ? ovv : load_f(L[I.a].ptr, L[I.a].dtype, off[I.a]); break;
      case AMC_OP_CONST: st[sp++] = I.imm; break;
      case AMC_OP_CVT: st[sp - 1] = round_f(I.a, st[sp - 1]); break;
      default:
        if (I.op < AMC_OP_ADD) st[sp - 1] = un_f(I.op, st[sp - 1]);
        else { st[sp - 2] = bin_f(I.op, st[sp - 2], st[sp - 1]); --sp; }
    }
  }
  return st[0];
}

// ------------------------------------------------------------------ map
template <bool ALLF>
__global__ void __launch_bounds__(256) k_map(const __grid_constant__ MapArgs a) {
  long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  long long stride = (long long)gridDim.x * blockDim.x;
  for (; i < a.total; i += stride) {
    long long off[kMaxLeaves];
    for (int l = 0; l < a.nleaf; ++l) off[l] = 0;
    long long rem = i;
    for (int d = a.rank - 1; d >= 0; --d) {
      long long s = a.shape[d];
      long long c = rem % s;
      rem /= s;
      for (int l = 0; l < a.nleaf; ++l) off[l] += c * a.leaf[l].strides[d];
    }
    if (ALLF) {
      double v = eval_prog_f(a.prog, a.leaf, off);
      store_num(a.out, a.out_dtype, i, nfl(v));
    } else {
      Num v = eval_prog(a.prog, a.leaf, off);
      store_num(a.out, a.out_dtype, i, v);
    }
  }
}

static unsigned grid_for(long long total, int block) {
  long long g = (total + block - 1) / block;
  long long cap = (long long)num_sms() * 16;
  if (g > cap) g = cap;
  if (g < 1) g = 1;
  return (unsigned)g;
}

// ------------------------------------------------------------------ view copies
// A pure copy (one leaf, same dtype) of a strided view in logical row-major
// order whose innermost axis is not the source's unit-stride axis while
// another axis t is (a transposed view): 32 x 32 tiles of (t, innermost) go
// through shared memory, so the reads run along t and the writes along the
// innermost output axis, both coalesced.  Values are copied bit for bit.
template <typename T>
__global__ void __launch_bounds__(256) k_copy_tiled(const __grid_constant__ MapArgs a, int t) {
  __shared__ T tile[32][33];
  const int r = a.rank, last = r - 1;
  const long long nt = a.shape[t], nl = a.shape[last];
  const long long tiles_l = (nl + 31) / 32, tiles_t = (nt + 31) / 32;
  long long ostr[AMC_MAX_RANK];
  long long acc = 1, batch = 1;
  for (int d = r - 1; d >= 0; --d) {
    ostr[d] = acc;
    acc *= a.shape[d];
    if (d != t && d != last) batch *= a.shape[d];
  }
  const T* src = (const T*)a.leaf[0].ptr;
  T* out = (T*)a.out;
  const long long st_t = a.leaf[0].strides[t], st_l = a.leaf[0].strides[last];
  const long long ntile = batch * tiles_t * tiles_l;
  for (long long tl = blockIdx.x; tl < ntile; tl += gridDim.x) {
    long long rem = tl;
    const long long il = rem % tiles_l;
    rem /= tiles_l;
    const long long it = rem % tiles_t;
    rem /= tiles_t;
    long long soff = 0, ooff = 0;
    for (int d = r - 1; d >= 0; --d) {
      if (d == t || d == last) continue;
      const long long c = rem % a.shape[d];
      rem /= a.shape[d];
      soff += c * a.leaf[0].strides[d];
      ooff += c * ostr[d];
    }
    const long long t0 = it * 32, l0 = il * 32;
    for (int k = threadIdx.y; k < 32; k += 8) {   // reads: threadIdx.x along t
      const long long ti = t0 + threadIdx.x, li = l0 + k;
      if (ti < nt && li < nl) tile[k][threadIdx.x] = src[soff + ti * st_t + li * st_l];
    }
    __syncthreads();
    for (int k = threadIdx.y; k < 32; k += 8) {   // writes: threadIdx.x along the innermost axis
      const long long ti = t0 + k, li = l0 + threadIdx.x;
      if (ti < nt && li < nl) out[ooff + ti * ostr[t] + li] = tile[threadIdx.x][k];
    }
    __syncthreads();
  }
}

// The unit-stride source axis of a pure same-dtype view copy that the tiled
// copy can take, or -1.
static int tiled_copy_axis(const MapArgs& a) {
  if (a.nleaf != 1 || a.rank < 2 || a.leaf[0].dtype != a.out_dtype) return -1;
  const bool load_only = a.prog.n == 1 && a.prog.code[0].op == AMC_OP_LOAD && a.prog.code[0].a == 0;
  const bool load_cvt_same = a.prog.n == 2 && a.prog.code[0].op == AMC_OP_LOAD && a.prog.code[0].a == 0 &&
                             a.prog.code[1].op == AMC_OP_CVT && a.prog.code[1].a == a.out_dtype;
  if (!load_only && !load_cvt_same) return -1;
  const int last = a.rank - 1;
  if (a.leaf[0].strides[last] == 1 || a.shape[last] < 2) return -1;
  for (int d = 0; d < last; ++d)
    if (a.leaf[0].strides[d] == 1 && a.shape[d] > 1) return d;
  return -1;
}

int launch_map(const MapArgs& a, cudaStream_t s) {
  if (a.total == 0) return AMC_OK;
  if (fault_injected("launch")) return fail(AMC_ERR_INJECTED, "map: injected launch failure (AMC_FAULT=launch)");
  const int t = tiled_copy_axis(a);
  if (t >= 0) {
    const int esz = dtype_size(a.out_dtype);
    const long long tiles = (a.total / (a.shape[t] * a.shape[a.rank - 1])) * ((a.shape[t] + 31) / 32) *
                            ((a.shape[a.rank - 1] + 31) / 32);
    // one tile per CTA where the grid allows: many resident CTAs hide the
    // load latency that each tile's barrier exposes
    const long long cap = 0x7fffffffLL;
    const unsigned g = (unsigned)(tiles < cap ? (tiles < 1 ? 1 : tiles) : cap);
    if (esz == 8) k_copy_tiled<unsigned long long><<<g, dim3(32, 8), 0, s>>>(a, t);
    else k_copy_tiled<unsigned int><<<g, dim3(32, 8), 0, s>>>(a, t);
    AMC_CUDA(cudaGetLastError());
    return AMC_OK;
  }
  unsigned g = grid_for(a.total, 256);
  if (a.prog.all_float) k_map<true><<<g, 256, 0, s>>>(a);
  else k_map<false><<<g, 256, 0, s>>>(a);
  AMC_CUDA(cudaGetLastError());
  return AMC_OK;
}

// ------------------------------------------------------------------ reductions
// Accumulator with the reference's reducer semantics: the running value is
// re-read from the typed output vector at every step, so it is rounded to
// the output dtype after each combination.
struct Acc {
  double f;
  long long i;
};

__device__ __forceinline__ void acc_init(Acc& A, int op, int out_dtype) {
  double v = op == AMC_RED_PROD ? 1.0 : op == AMC_RED_MAX ? -INFINITY : op == AMC_RED_MIN ? INFINITY : 0.0;
  A.f = v;
  A.i = op == AMC_RED_PROD ? 1 : 0;
}

// src values are either all exact (integer source dtype) or all inexact.
__device__ __forceinline__ void acc_step(Acc& A, int op, int out_dtype, bool src_exact, double vf, long long vi) {
  if (dtype_is_float_d(out_dtype)) {
    double x = src_exact ? (double)vi : vf;
    double r;
    switch (op) {
      case AMC_RED_PROD: r = __dmul_rn(A.f, x); break;
      case AMC_RED_MAX: r = A.f > x ? A.f : x; break;  // (max acc x): acc kept only when strictly larger
      case AMC_RED_MIN: r = A.f < x ? A.f : x; break;
      default: r = __dadd_rn(A.f, x); break;
    }
    A.f = out_dtype == AMC_F32 ? (double)__double2float_rn(r) : r;
  } else {
    long long r = op == AMC_RED_PROD ? A.i * vi : A.i + vi;
    switch (out_dtype) {
      case AMC_S32: r = (int)r; break;
      case AMC_U32: r = (unsigned)(r < 0 ? -r : r); break;
      case AMC_U64: r = r < 0 ? -r : r; break;
      default: break;
    }
    A.i = r;
  }
}

__device__ __forceinline__ void acc_store(const Acc& A, void* out, int out_dtype, int op, long long R, long long o) {
  if (dtype_is_float_d(out_dtype)) {
    double v = A.f;
    if (op == AMC_RED_MEAN) v = __ddiv_rn(v, (double)R);
    store_num(out, out_dtype, o, nfl(v));
  } else {
    store_num(out, out_dtype, o, nex(A.i));
  }
}

__device__ __forceinline__ void leaf_offsets(const ReduceArgs& a, long long o, long long r, long long* off) {
  if (a.orank == 1 && a.rrank == 1) {   // one kept and one reduced axis: no index decomposition
    for (int l = 0; l < a.nleaf; ++l) off[l] = o * a.leaf_o[l].strides[0] + r * a.leaf_r[l][0];
    return;
  }
  if (a.orank == 0 && a.rrank == 1) {   // a full reduction of one axis
    for (int l = 0; l < a.nleaf; ++l) off[l] = r * a.leaf_r[l][0];
    return;
  }
  for (int l = 0; l < a.nleaf; ++l) off[l] = 0;
  long long rem = o;
  for (int d = a.orank - 1; d >= 0; --d) {
    long long s = a.oshape[d], c = rem % s;
    rem /= s;
    for (int l = 0; l < a.nleaf; ++l) off[l] += c * a.leaf_o[l].strides[d];
  }
  rem = r;
  for (int d = a.rrank - 1; d >= 0; --d) {
    long long s = a.rshape[d], c = rem % s;
    rem /= s;
    for (int l = 0; l < a.nleaf; ++l) off[l] += c * a.leaf_r[l][d];
  }
}

// Evaluate the source element (o, r): the value after the source node's store
// conversion, returned as (double, int64) by the source dtype's exactness.
__device__ __forceinline__ void eval_src(const ReduceArgs& a, long long o, long long r, double& vf, long long& vi) {
  long long off[kMaxLeaves];
  leaf_offsets(a, o, r, off);
  if (a.prog.all_float) {
    vf = eval_prog_f(a.prog, a.leaf_o, off);
    vi = 0;
  } else {
    Num v = eval_prog(a.prog, a.leaf_o, off);
    vf = as_f(v);
    vi = trunc_i(v);
  }
}

// Ordered ("sequential") reduction: CTA owns OT consecutive outputs.  All
// threads evaluate a (OT x RC) tile of source values into shared memory in
// parallel; then one thread per output folds its RC values in ascending r.
// This reproduces the reference's accumulation order exactly.  The fold is
// one dependent chain per output, so its step is specialised (`fold`):
//   1 sum/mean into f64 from an inexact source, 2 the same into f32 (rounded
//   to f32 after every step, as the reference's typed output is re-read),
//   3 sum/mean into s32/s64 from an exact source, 4 sum/mean of f32 values
//   into f32; 0 the generic step.  Fold 4 adds in f32 directly: for f32 a
//   and b, rounding the double sum to f32 gives the f32-rounded sum, because
//   double has more than 2 x 24 + 2 significand bits.  The f32 add is a
//   4-clock chain step; the double add followed by the f32 conversion
//   measured 46.
template <int FOLD>
__device__ __forceinline__ void fold_row(Acc& A, int op, int out_dtype, bool src_exact,
                                         const unsigned long long* __restrict__ row, int rc) {
  if (FOLD == 1) {
    double acc = A.f;
#pragma unroll 8
    for (int rl = 0; rl < rc; ++rl) acc = __dadd_rn(acc, __longlong_as_double(row[rl]));
    A.f = acc;
  } else if (FOLD == 2) {
    double acc = A.f;
#pragma unroll 8
    for (int rl = 0; rl < rc; ++rl) acc = (double)__double2float_rn(__dadd_rn(acc, __longlong_as_double(row[rl])));
    A.f = acc;
  } else if (FOLD == 3) {
    long long acc = A.i;
    if (out_dtype == AMC_S32) {
#pragma unroll 8
      for (int rl = 0; rl < rc; ++rl) acc = (int)(acc + (long long)row[rl]);
    } else {
#pragma unroll 8
      for (int rl = 0; rl < rc; ++rl) acc += (long long)row[rl];
    }
    A.i = acc;
  } else if (FOLD == 4) {
    float acc = (float)A.f;
#pragma unroll 8
    for (int rl = 0; rl < rc; ++rl) acc = __fadd_rn(acc, (float)__longlong_as_double(row[rl]));
    A.f = (double)acc;
  } else {
    for (int rl = 0; rl < rc; ++rl) {
      unsigned long long bits = row[rl];
      acc_step(A, op, out_dtype, src_exact, __longlong_as_double(bits), (long long)bits);
    }
  }
}

// Small float programs (at most 2 leaves, stack depth at most 3) of a
// reduction over one kept and one reduced axis: the source values of kSmallV
// elements are gathered first (all loads in flight together: the cost of an
// element is one memory latency, not one per LOAD instruction), then the
// program runs on named registers: the leaf values and the three stack slots
// are selected by switches on warp-uniform indices, so nothing goes to local
// memory.  Values and rounding are those of eval_prog_f.
constexpr int kSmallV = 4;

__device__ __forceinline__ double small_unary(int op, int cvt, double x) {
  if (op == AMC_OP_CVT) return cvt == AMC_F64 ? x : cvt == AMC_F32 ? (double)__double2float_rn(x) : round_f(cvt, x);
  return un_f(op, x);
}

__device__ __forceinline__ void eval_small_vals(const DProg& P, const double (&l0)[kSmallV], const double (&l1)[kSmallV],
                                                double (&out)[kSmallV]);

__device__ __forceinline__ void eval_small(const ReduceArgs& a, const long long (&o)[kSmallV],
                                           const long long (&r)[kSmallV], double (&out)[kSmallV]) {
  double l0[kSmallV], l1[kSmallV];
#pragma unroll
  for (int v = 0; v < kSmallV; ++v) {
    l0[v] = load_f(a.leaf_o[0].ptr, a.leaf_o[0].dtype, o[v] * a.leaf_o[0].strides[0] + r[v] * a.leaf_r[0][0]);
    l1[v] = a.nleaf > 1
                ? load_f(a.leaf_o[1].ptr, a.leaf_o[1].dtype, o[v] * a.leaf_o[1].strides[0] + r[v] * a.leaf_r[1][0])
                : 0.0;
  }
  eval_small_vals(a.prog, l0, l1, out);
}

// The small program on gathered leaf values (l0: leaf 0, l1: leaf 1).
__device__ __forceinline__ void eval_small_vals(const DProg& P, const double (&l0)[kSmallV], const double (&l1)[kSmallV],
                                                double (&out)[kSmallV]) {
#pragma unroll
  for (int v = 0; v < kSmallV; ++v) {
    double s0 = 0.0, s1 = 0.0, s2 = 0.0;
    int sp = 0;
    for (int pc = 0; pc < P.n; ++pc) {
      const amc_insn I = P.code[pc];
      if (I.op == AMC_OP_LOAD || I.op == AMC_OP_CONST) {
        const double t = I.op == AMC_OP_CONST ? I.imm : (I.a == 0 ? l0[v] : l1[v]);
        if (sp == 0) s0 = t;
        else if (sp == 1) s1 = t;
        else s2 = t;
        ++sp;
      } else if (I.op < AMC_OP_ADD) {
        if (sp == 1) s0 = small_unary(I.op, I.a, s0);
        else if (sp == 2) s1 = small_unary(I.op, I.a, s1);
        else s2 = small_unary(I.op, I.a, s2);
      } else {
        if (sp == 2) s0 = bin_f(I.op, s0, s1);
        else s1 = bin_f(I.op, s1, s2);
        --sp;
      }
    }
    out[v] = s0;
  }
}

template <int FOLD>
__global__ void __launch_bounds__(256, 4) k_reduce_seq(const __grid_constant__ ReduceArgs a, int OT, int RC, int ofast) {
  extern __shared__ unsigned long long smem_u64[];
  const bool src_exact = !dtype_is_float_d(a.src_dtype);
  const bool small = a.prog.all_float && a.prog.max_depth <= 3 && a.nleaf <= 2 && a.orank == 1 && a.rrank == 1;
  const long long o0 = (long long)blockIdx.x * OT;
  Acc A;
  acc_init(A, a.op, a.out_dtype);
  for (long long r0 = 0; r0 < a.R; r0 += RC) {
    int rc = (int)((a.R - r0) < RC ? (a.R - r0) : RC);
    int tile = OT * rc;
    if (small) {
      for (int e0 = threadIdx.x; e0 < tile; e0 += blockDim.x * kSmallV) {
        long long oo[kSmallV], rr[kSmallV];
        int slot[kSmallV];
#pragma unroll
        for (int k = 0; k < kSmallV; ++k) {
          const int e = e0 + k * blockDim.x;
          int ol = 0, rl = 0;
          if (ofast) { ol = e % OT; rl = e / OT; } else { ol = e / rc; rl = e % rc; }
          const bool valid = e < tile && o0 + ol < a.O;
          slot[k] = valid ? ol * (RC + 1) + rl : -1;
          oo[k] = valid ? o0 + ol : 0;   // element (0, 0) of every leaf: in bounds, unused
          rr[k] = valid ? r0 + rl : 0;
        }
        double v[kSmallV];
        eval_small(a, oo, rr, v);
#pragma unroll
        for (int k = 0; k < kSmallV; ++k)
          if (slot[k] >= 0) smem_u64[slot[k]] = __double_as_longlong(v[k]);
      }
    } else {
      for (int e = threadIdx.x; e < tile; e += blockDim.x) {
        int ol, rl;
        if (ofast) { ol = e % OT; rl = e / OT; } else { ol = e / rc; rl = e % rc; }
        long long o = o0 + ol;
        if (o >= a.O) continue;
        double vf; long long vi;
        eval_src(a, o, r0 + rl, vf, vi);
        smem_u64[ol * (RC + 1) + rl] = src_exact ? (unsigned long long)vi : __double_as_longlong(vf);
      }
    }
    __syncthreads();
    if (threadIdx.x < OT && o0 + threadIdx.x < a.O)
      fold_row<FOLD>(A, a.op, a.out_dtype, src_exact, smem_u64 + threadIdx.x * (RC + 1), rc);
    __syncthreads();
  }
  if (threadIdx.x < OT && o0 + threadIdx.x < a.O) acc_store(A, a.out, a.out_dtype, a.op, a.R, o0 + threadIdx.x);
}

// Staged ordered reduction for one kept and one reduced axis with outputs
// adjacent in memory and a small program (at most 2 leaves, stack depth 3),
// float or exact.  k_reduce_seq gives each CTA only a couple of outputs when
// there are few of them, so every warp load uses a fraction of a 32-byte
// sector from many rows and the L2 request rate, not bandwidth, bounds the
// gather.  Here a CTA owns OT (8) consecutive outputs, so a warp load covers
// whole sectors, and the raw leaf values of the whole (OT x rc) tile are
// copied into shared memory with cp.async, all in flight at once and holding
// no registers.  The program then runs from shared memory (values and
// rounding as eval_prog / eval_prog_f), and the fold is the same ascending
// chain as k_reduce_seq, with its shared loads issued a batch ahead.
__device__ __forceinline__ void cp_async_elem(void* dst, const void* src, int bytes) {
  if (bytes == 8)
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)), "l"(src) : "memory");
  else
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
// Named barrier over `count` threads (whole warps).
__device__ __forceinline__ void named_bar(int id, int count) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory"); }
__device__ __forceinline__ int dtype_bytes_d(int d) { return (d == AMC_F32 || d == AMC_S32 || d == AMC_U32) ? 4 : 8; }

__device__ __forceinline__ double raw_f(unsigned long long raw, int dtype) {
  return dtype == AMC_F32 ? (double)__int_as_float((int)(unsigned)raw) : __longlong_as_double((long long)raw);
}
__device__ __forceinline__ Num raw_num(unsigned long long raw, int dtype) {
  switch (dtype) {
    case AMC_F32: return nfl((double)__int_as_float((int)(unsigned)raw));
    case AMC_F64: return nfl(__longlong_as_double((long long)raw));
    case AMC_S32: return nex((long long)(int)(unsigned)raw);
    case AMC_U32: return nex((long long)(unsigned)raw);
    default: return nex((long long)raw);
  }
}

// One element of a small program on named registers (stack slots s0..s2).
template <bool EXACT>
__device__ __forceinline__ void eval_staged(const amc_insn* code, int n, const DLeaf* L, unsigned long long r0,
                                            unsigned long long r1, double& vf, long long& vi) {
  if (!EXACT) {
    const double l0 = raw_f(r0, L[0].dtype), l1 = raw_f(r1, L[1].dtype);
    double s0 = 0.0, s1 = 0.0, s2 = 0.0;
    int sp = 0;
    for (int pc = 0; pc < n; ++pc) {
      const amc_insn I = code[pc];
      if (I.op == AMC_OP_LOAD || I.op == AMC_OP_CONST) {
        const double t = I.op == AMC_OP_CONST ? I.imm : (I.a == 0 ? l0 : l1);
        if (sp == 0) s0 = t;
        else if (sp == 1) s1 = t;
        else s2 = t;
        ++sp;
      } else if (I.op < AMC_OP_ADD) {
        if (sp == 1) s0 = small_unary(I.op, I.a, s0);
        else if (sp == 2) s1 = small_unary(I.op, I.a, s1);
        else s2 = small_unary(I.op, I.a, s2);
      } else {
        if (sp == 2) s0 = bin_f(I.op, s0, s1);
        else s1 = bin_f(I.op, s1, s2);
        --sp;
      }
    }
    vf = s0;
    vi = 0;
  } else {
    const Num l0 = raw_num(r0, L[0].dtype), l1 = raw_num(r1, L[1].dtype);
    Num s0 = nex(0), s1 = nex(0), s2 = nex(0);
    int sp = 0;
    for (int pc = 0; pc < n; ++pc) {
      const amc_insn I = code[pc];
      if (I.op == AMC_OP_LOAD || I.op == AMC_OP_CONST || I.op == AMC_OP_ICONST) {
        const Num t = I.op == AMC_OP_CONST ? nfl(I.imm) : I.op == AMC_OP_ICONST ? nex((long long)I.imm) : (I.a == 0 ? l0 : l1);
        if (sp == 0) s0 = t;
        else if (sp == 1) s1 = t;
        else s2 = t;
        ++sp;
      } else if (I.op == AMC_OP_CVT) {
        if (sp == 1) s0 = round_store(I.a, s0);
        else if (sp == 2) s1 = round_store(I.a, s1);
        else s2 = round_store(I.a, s2);
      } else if (I.op < AMC_OP_ADD) {
        if (sp == 1) s0 = un_op(I.op, s0);
        else if (sp == 2) s1 = un_op(I.op, s1);
        else s2 = un_op(I.op, s2);
      } else {
        if (sp == 2) s0 = bin_op(I.op, s0, s1);
        else s1 = bin_op(I.op, s1, s2);
        --sp;
      }
    }
    vf = as_f(s0);
    vi = trunc_i(s0);
  }
}

// fold of one output row with the shared loads issued a batch of 8 ahead of
// the dependent additions (same order and rounding as fold_row)
template <int FOLD>
__device__ __forceinline__ void fold_row_pipelined(Acc& A, int op, int out_dtype, bool src_exact,
                                                   const unsigned long long* __restrict__ row, int rc) {
  if (FOLD == 0) {
    fold_row<0>(A, op, out_dtype, src_exact, row, rc);
    return;
  }
  constexpr int B = 8;
  unsigned long long cur[B], nxt[B];
  int rl = 0;
  if (rc >= B) {
#pragma unroll
    for (int k = 0; k < B; ++k) cur[k] = row[k];
  }
  for (; rl + B <= rc; rl += B) {
    const bool more = rl + 2 * B <= rc;
    if (more) {
#pragma unroll
      for (int k = 0; k < B; ++k) nxt[k] = row[rl + B + k];
    }
    if (FOLD == 1) {
      double acc = A.f;
#pragma unroll
      for (int k = 0; k < B; ++k) acc = __dadd_rn(acc, __longlong_as_double(cur[k]));
      A.f = acc;
    } else if (FOLD == 4) {
      float acc = (float)A.f;
#pragma unroll
      for (int k = 0; k < B; ++k) acc = __fadd_rn(acc, (float)__longlong_as_double(cur[k]));
      A.f = (double)acc;
    } else if (FOLD == 2) {
      double acc = A.f;
#pragma unroll
      for (int k = 0; k < B; ++k) acc = (double)__double2float_rn(__dadd_rn(acc, __longlong_as_double(cur[k])));
      A.f = acc;
    } else if (out_dtype == AMC_S32) {
      // truncation to 32 bits commutes with addition, so a 32-bit wrapping
      // sum equals truncating the 64-bit sum after every step
      unsigned acc = (unsigned)A.i;
#pragma unroll
      for (int k = 0; k < B; ++k) acc += (unsigned)cur[k];
      A.i = (long long)(int)acc;
    } else {
      long long acc = A.i;
#pragma unroll
      for (int k = 0; k < B; ++k) acc += (long long)cur[k];
      A.i = acc;
    }
    if (more) {
#pragma unroll
      for (int k = 0; k < B; ++k) cur[k] = nxt[k];
    }
  }
  if (rl < rc) fold_row<FOLD>(A, op, out_dtype, src_exact, row + rl, rc - rl);
}

// V elements per dispatch of each program instruction: the op and stack-slot
// switches run once for V independent elements, which also gives the V
// dependent chains instruction-level parallelism.  Values and rounding are
// those of eval_prog_f (float programs) and eval_prog (integer-only programs:
// integer leaves, ICONST, integer stores, NEG ABS ADD SUB MUL MAX MIN, where
// every value stays exact).
template <int V>
__device__ __forceinline__ void vec_push_f(double (&d)[V], const amc_insn& I, const double (&l0)[V], const double (&l1)[V]) {
#pragma unroll
  for (int k = 0; k < V; ++k) d[k] = I.op == AMC_OP_CONST ? I.imm : (I.a == 0 ? l0[k] : l1[k]);
}
template <int V>
__device__ __forceinline__ void vec_unary_f(int op, int cvt, double (&t)[V]) {
  switch (op) {
    case AMC_OP_CVT:
      if (cvt == AMC_F64) break;
      if (cvt == AMC_F32) {
#pragma unroll
        for (int k = 0; k < V; ++k) t[k] = (double)__double2float_rn(t[k]);
        break;
      }
#pragma unroll
      for (int k = 0; k < V; ++k) t[k] = round_f(cvt, t[k]);
      break;
    case AMC_OP_NEG:
#pragma unroll
      for (int k = 0; k < V; ++k) t[k] = -t[k];
      break;
    case AMC_OP_ABS:
#pragma unroll
      for (int k = 0; k < V; ++k) t[k] = fabs(t[k]);
      break;
    default:
#pragma unroll
      for (int k = 0; k < V; ++k) t[k] = un_f(op, t[k]);
  }
}
template <int V>
__device__ __forceinline__ void vec_binary_f(int op, double (&x)[V], const double (&y)[V]) {
  switch (op) {
    case AMC_OP_ADD:
#pragma unroll
      for (int k = 0; k < V; ++k) x[k] = __dadd_rn(x[k], y[k]);
      break;
    case AMC_OP_SUB:
#pragma unroll
      for (int k = 0; k < V; ++k) x[k] = __dsub_rn(x[k], y[k]);
      break;
    case AMC_OP_MUL:
#pragma unroll
      for (int k = 0; k < V; ++k) x[k] = __dmul_rn(x[k], y[k]);
      break;
    default:
#pragma unroll
      for (int k = 0; k < V; ++k) x[k] = bin_f(op, x[k], y[k]);
  }
}
template <int V>
__device__ __forceinline__ void eval_vec_f(const amc_insn* code, int n, const double (&l0)[V], const double (&l1)[V],
                                           double (&out)[V]) {
  double s0[V], s1[V], s2[V];
  int sp = 0;
  for (int pc = 0; pc < n; ++pc) {
    const amc_insn I = code[pc];
    if (I.op == AMC_OP_LOAD || I.op == AMC_OP_CONST) {
      if (sp == 0) vec_push_f(s0, I, l0, l1);
      else if (sp == 1) vec_push_f(s1, I, l0, l1);
      else vec_push_f(s2, I, l0, l1);
      ++sp;
    } else if (I.op < AMC_OP_ADD) {
      if (sp == 1) vec_unary_f(I.op, I.a, s0);
      else if (sp == 2) vec_unary_f(I.op, I.a, s1);
      else vec_unary_f(I.op, I.a, s2);
    } else {
      if (sp == 2) vec_binary_f(I.op, s0, s1);
      else vec_binary_f(I.op, s1, s2);
      --sp;
    }
  }
#pragma unroll
  for (int k = 0; k < V; ++k) out[k] = s0[k];
}

template <int V>
__device__ __forceinline__ void vec_push_i(long long (&d)[V], const amc_insn& I, const long long (&l0)[V],
                                           const long long (&l1)[V]) {
#pragma unroll
  for (int k = 0; k < V; ++k) d[k] = I.op == AMC_OP_ICONST ? (long long)I.imm : (I.a == 0 ? l0[k] : l1[k]);
}
__device__ __forceinline__ long long store_int(int dtype, long long t) {
  switch (dtype) {
    case AMC_S32: return (int)t;
    case AMC_U32: return (unsigned)(t < 0 ? -t : t);
    case AMC_U64: return t < 0 ? -t : t;
    default: return t;
  }
}
template <int V>
__device__ __forceinline__ void vec_unary_i(int op, int cvt, long long (&t)[V]) {
  switch (op) {
    case AMC_OP_CVT:
      if (cvt == AMC_S32) {
#pragma unroll
        for (int k = 0; k < V; ++k) t[k] = (int)t[k];
      } else if (cvt != AMC_S64) {
#pragma unroll
        for (int k = 0; k < V; ++k) t[k] = store_int(cvt, t[k]);
      }
      break;
    case AMC_OP_NEG:
#pragma unroll
      for (int k = 0; k < V; ++k) t[k] = -t[k];
      break;
    default:   // ABS
#pragma unroll
      for (int k = 0; k < V; ++k) t[k] = t[k] < 0 ? -t[k] : t[k];
  }
}
template <int V>
__device__ __forceinline__ void vec_binary_i(int op, long long (&x)[V], const long long (&y)[V]) {
  switch (op) {
    case AMC_OP_ADD:
#pragma unroll
      for (int k = 0; k < V; ++k) x[k] = x[k] + y[k];
      break;
    case AMC_OP_SUB:
#pragma unroll
      for (int k = 0; k < V; ++k) x[k] = x[k] - y[k];
      break;
    case AMC_OP_MUL:
#pragma unroll
      for (int k = 0; k < V; ++k) x[k] = x[k] * y[k];
      break;
    case AMC_OP_MAX:
#pragma unroll
      for (int k = 0; k < V; ++k) x[k] = x[k] > y[k] ? x[k] : y[k];
      break;
    default:   // MIN
#pragma unroll
      for (int k = 0; k < V; ++k) x[k] = x[k] < y[k] ? x[k] : y[k];
  }
}
template <int V>
__device__ __forceinline__ void eval_vec_i(const amc_insn* code, int n, const long long (&l0)[V],
                                           const long long (&l1)[V], long long (&out)[V]) {
  long long s0[V], s1[V], s2[V];
  int sp = 0;
  for (int pc = 0; pc < n; ++pc) {
    const amc_insn I = code[pc];
    if (I.op == AMC_OP_LOAD || I.op == AMC_OP_ICONST) {
      if (sp == 0) vec_push_i(s0, I, l0, l1);
      else if (sp == 1) vec_push_i(s1, I, l0, l1);
      else vec_push_i(s2, I, l0, l1);
      ++sp;
    } else if (I.op < AMC_OP_ADD) {
      if (sp == 1) vec_unary_i(I.op, I.a, s0);
      else if (sp == 2) vec_unary_i(I.op, I.a, s1);
      else vec_unary_i(I.op, I.a, s2);
    } else {
      if (sp == 2) vec_binary_i(I.op, s0, s1);
      else vec_binary_i(I.op, s1, s2);
      --sp;
    }
  }
#pragma unroll
  for (int k = 0; k < V; ++k) out[k] = s0[k];
}
__device__ __forceinline__ long long raw_i(unsigned long long raw, int dtype) {
  switch (dtype) {
    case AMC_S32: return (long long)(int)(unsigned)raw;
    case AMC_U32: return (long long)(unsigned)raw;
    default: return (long long)raw;
  }
}

// Host check: the program keeps every value an exact integer (eval_vec_i).
static bool prog_int_only(const ReduceArgs& a) {
  for (int l = 0; l < a.nleaf; ++l)
    if (a.leaf_o[l].dtype == AMC_F32 || a.leaf_o[l].dtype == AMC_F64) return false;
  for (int pc = 0; pc < a.prog.n; ++pc) {
    const amc_insn& I = a.prog.code[pc];
    switch (I.op) {
      case AMC_OP_LOAD: case AMC_OP_ICONST: case AMC_OP_NEG: case AMC_OP_ABS: case AMC_OP_ADD: case AMC_OP_SUB:
      case AMC_OP_MUL: case AMC_OP_MAX: case AMC_OP_MIN:
        break;
      case AMC_OP_CVT:
        if (I.a == AMC_F32 || I.a == AMC_F64) return false;
        break;
      default:
        return false;
    }
  }
  return true;
}

constexpr int kStOT = 4;          // outputs per CTA (4 f64 = one 32-byte sector)
constexpr int kStSC = 192;        // reduced positions per sub-chunk (static shared memory < 48 KB)
constexpr int kStWorkers = 224;   // warps 1-7 copy and evaluate; warp 0 folds

template <int MODE, int V>
__device__ __forceinline__ void staged_eval_chunk(const ReduceArgs& a, const amc_insn* code,
                                                  const unsigned long long* __restrict__ raw0,
                                                  const unsigned long long* __restrict__ raw1,
                                                  unsigned long long* __restrict__ vals, long long o0, int tile,
                                                  int wt, bool src_exact) {
  const int nl = a.nleaf;
  const int dt0 = a.leaf_o[0].dtype, dt1 = nl > 1 ? a.leaf_o[1].dtype : dt0;
  for (int e0 = wt; e0 < tile; e0 += kStWorkers * V) {
    int slot[V];
#pragma unroll
    for (int k = 0; k < V; ++k) {
      const int e = e0 + k * kStWorkers;
      const bool valid = e < tile && o0 + (e & (kStOT - 1)) < a.O;
      slot[k] = valid ? (e & (kStOT - 1)) * (kStSC + 1) + e / kStOT : -1;
    }
    if (MODE == 0) {
      double l0[V], l1[V], out[V];
#pragma unroll
      for (int k = 0; k < V; ++k) {
        const int e = e0 + k * kStWorkers;
        l0[k] = slot[k] >= 0 ? raw_f(raw0[e], dt0) : 0.0;
        l1[k] = (slot[k] >= 0 && nl > 1) ? raw_f(raw1[e], dt1) : 0.0;
      }
      eval_vec_f<V>(code, a.prog.n, l0, l1, out);
#pragma unroll
      for (int k = 0; k < V; ++k)
        if (slot[k] >= 0)
          vals[slot[k]] = src_exact ? (unsigned long long)(long long)trunc(out[k])
                                    : (unsigned long long)__double_as_longlong(out[k]);
    } else if (MODE == 1) {
      long long l0[V], l1[V], out[V];
#pragma unroll
      for (int k = 0; k < V; ++k) {
        const int e = e0 + k * kStWorkers;
        l0[k] = slot[k] >= 0 ? raw_i(raw0[e], dt0) : 0;
        l1[k] = (slot[k] >= 0 && nl > 1) ? raw_i(raw1[e], dt1) : 0;
      }
      eval_vec_i<V>(code, a.prog.n, l0, l1, out);
#pragma unroll
      for (int k = 0; k < V; ++k)
        if (slot[k] >= 0)
          vals[slot[k]] = src_exact ? (unsigned long long)out[k]
                                    : (unsigned long long)__double_as_longlong((double)out[k]);
    } else {
#pragma unroll
      for (int k = 0; k < V; ++k) {
        if (slot[k] < 0) continue;
        const int e = e0 + k * kStWorkers;
        double vf;
        long long vi;
        eval_staged<true>(code, a.prog.n, a.leaf_o, raw0[e], nl > 1 ? raw1[e] : 0ull, vf, vi);
        vals[slot[k]] = src_exact ? (unsigned long long)vi : (unsigned long long)__double_as_longlong(vf);
      }
    }
  }
}

template <int FOLD, int MODE>
__global__ void __launch_bounds__(256) k_reduce_staged(const __grid_constant__ ReduceArgs a) {
  __shared__ unsigned long long raw[2][2][kStOT * kStSC];        // [buffer][leaf][position][output]
  __shared__ unsigned long long vals[2][kStOT * (kStSC + 1)];    // [buffer][output][position]
  __shared__ amc_insn code[AMC_PROG_MAX];   // the program, read by every evaluation step
  const int tid = threadIdx.x;
  for (int i = tid; i < a.prog.n; i += blockDim.x) code[i] = a.prog.code[i];
  __syncthreads();
  const bool src_exact = !dtype_is_float_d(a.src_dtype);
  const long long o0 = (long long)blockIdx.x * kStOT;
  const int nch = (int)((a.R + kStSC - 1) / kStSC);
  if (tid < 32) {
    // fold warp: sub-chunk j once the workers have evaluated it
    Acc A;
    acc_init(A, a.op, a.out_dtype);
    for (int j = 0; j < nch; ++j) {
      named_bar(2, 256);
      const int rc = (int)((a.R - (long long)j * kStSC) < kStSC ? (a.R - (long long)j * kStSC) : kStSC);
      if (tid < kStOT && o0 + tid < a.O)
        fold_row_pipelined<FOLD>(A, a.op, a.out_dtype, src_exact, vals[j & 1] + tid * (kStSC + 1), rc);
    }
    if (tid < kStOT && o0 + tid < a.O) acc_store(A, a.out, a.out_dtype, a.op, a.R, o0 + tid);
    return;
  }
  // workers: copy sub-chunk j+1 (cp.async, outputs fastest so a warp covers
  // whole sectors) while evaluating sub-chunk j
  const int wt = tid - 32;
  const int nl = a.nleaf;
  const int b0 = dtype_bytes_d(a.leaf_o[0].dtype), b1 = nl > 1 ? dtype_bytes_d(a.leaf_o[1].dtype) : 8;
  const char* p0 = (const char*)a.leaf_o[0].ptr;
  const char* p1 = nl > 1 ? (const char*)a.leaf_o[1].ptr : p0;
  const long long so0 = a.leaf_o[0].strides[0], sr0 = a.leaf_r[0][0];
  const long long so1 = nl > 1 ? a.leaf_o[1].strides[0] : 0, sr1 = nl > 1 ? a.leaf_r[1][0] : 0;
  auto copy = [&](int j) {
    const long long r0 = (long long)j * kStSC;
    const int rc = (int)((a.R - r0) < kStSC ? (a.R - r0) : kStSC);
    const int tile = kStOT * rc;
    unsigned long long* d0 = raw[j & 1][0];
    unsigned long long* d1 = raw[j & 1][1];
    for (int e = wt; e < tile; e += kStWorkers) {
      const long long o = o0 + (e & (kStOT - 1));
      if (o >= a.O) continue;
      const long long r = r0 + e / kStOT;
      cp_async_elem(d0 + e, p0 + (o * so0 + r * sr0) * b0, b0);
      if (nl > 1) cp_async_elem(d1 + e, p1 + (o * so1 + r * sr1) * b1, b1);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  copy(0);
  for (int j = 0; j < nch; ++j) {
    if (j + 1 < nch) {
      copy(j + 1);
      asm volatile("cp.async.wait_group 1;" ::: "memory");
    } else {
      asm volatile("cp.async.wait_group 0;" ::: "memory");
    }
    named_bar(1, kStWorkers);   // sub-chunk j has landed for every worker
    const long long r0 = (long long)j * kStSC;
    const int rc = (int)((a.R - r0) < kStSC ? (a.R - r0) : kStSC);
    staged_eval_chunk<MODE, 4>(a, code, raw[j & 1][0], raw[j & 1][1], vals[j & 1], o0, kStOT * rc, wt, src_exact);
    // hand sub-chunk j to the fold warp; it arrives here after folding j-1,
    // so vals[j & 1] is free again from the next iteration on
    named_bar(2, 256);
  }
}

// Tree reduction for few outputs over long axes: pass 1 gives each CTA of
// grid (G, O) a contiguous r-range, folded per thread in ascending order and
// combined across the block in a fixed tree; pass 2 folds the G partials of
// each output in ascending order.  Deterministic; float sums accumulate in
// double (tighter than the reference's running f32 sum).
__device__ __forceinline__ void tree_combine(int op, bool exact, double& f, long long& i, double f2, long long i2) {
  if (exact) {
    i = op == AMC_RED_PROD ? i * i2 : i + i2;
  } else {
    switch (op) {
      case AMC_RED_PROD: f = f * f2; break;
      case AMC_RED_MAX: f = f2 > f ? f2 : f; break;
      case AMC_RED_MIN: f = f2 < f ? f2 : f; break;
      default: f = f + f2; break;
    }
  }
}

__global__ void __launch_bounds__(256) k_reduce_tree1(const __grid_constant__ ReduceArgs a, double* pf, long long* pi, int G) {
  const bool exact = !dtype_is_float_d(a.src_dtype);
  const int g = blockIdx.x;
  const long long o = blockIdx.y;
  long long chunk = (a.R + G - 1) / G, r_begin = g * chunk, r_end = r_begin + chunk < a.R ? r_begin + chunk : a.R;
  double f = a.op == AMC_RED_PROD ? 1.0 : a.op == AMC_RED_MAX ? -INFINITY : a.op == AMC_RED_MIN ? INFINITY : 0.0;
  long long i = a.op == AMC_RED_PROD ? 1 : 0;
  long long r = r_begin + threadIdx.x;
  if (a.prog.all_float && a.prog.max_depth <= 3 && a.nleaf <= 2) {
    // small float programs: the leaves of kSmallV elements gathered together
    // (one memory latency per kSmallV elements), the program on registers;
    // each thread still combines its elements in ascending r
    const long long step = (long long)blockDim.x;
    for (; r + (kSmallV - 1) * step < r_end; r += kSmallV * step) {
      double l0[kSmallV], l1[kSmallV], v[kSmallV];
#pragma unroll
      for (int k = 0; k < kSmallV; ++k) {
        long long off[kMaxLeaves];
        leaf_offsets(a, o, r + k * step, off);
        l0[k] = load_f(a.leaf_o[0].ptr, a.leaf_o[0].dtype, off[0]);
        l1[k] = a.nleaf > 1 ? load_f(a.leaf_o[1].ptr, a.leaf_o[1].dtype, off[1]) : 0.0;
      }
      eval_small_vals(a.prog, l0, l1, v);
#pragma unroll
      for (int k = 0; k < kSmallV; ++k) tree_combine(a.op, false, f, i, v[k], 0);
    }
  }
  for (; r < r_end; r += blockDim.x) {
    double vf; long long vi;
    eval_src(a, o, r, vf, vi);
    tree_combine(a.op, exact, f, i, vf, vi);
  }
  __shared__ double sf[256];
  __shared__ long long si[256];
  sf[threadIdx.x] = f;
  si[threadIdx.x] = i;
  __syncthreads();
  for (int w = blockDim.x / 2; w > 0; w >>= 1) {
    if (threadIdx.x < w) {
      double f2 = sf[threadIdx.x + w]; long long i2 = si[threadIdx.x + w];
      double f1 = sf[threadIdx.x]; long long i1 = si[threadIdx.x];
      tree_combine(a.op, exact, f1, i1, f2, i2);
      sf[threadIdx.x] = f1; si[threadIdx.x] = i1;
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) { pf[o * G + g] = sf[0]; pi[o * G + g] = si[0]; }
}

// Pass 2: one CTA per output; thread t folds partials t, t+128, ... in
// ascending order, then the 128 folds combine in a fixed tree.
__global__ void __launch_bounds__(128) k_reduce_tree2(const __grid_constant__ ReduceArgs a, const double* pf,
                                                      const long long* pi, int G) {
  const long long o = blockIdx.x;
  const bool exact = !dtype_is_float_d(a.src_dtype);
  double f = a.op == AMC_RED_PROD ? 1.0 : a.op == AMC_RED_MAX ? -INFINITY : a.op == AMC_RED_MIN ? INFINITY : 0.0;
  long long i = a.op == AMC_RED_PROD ? 1 : 0;
  for (int g = threadIdx.x; g < G; g += blockDim.x) tree_combine(a.op, exact, f, i, pf[o * G + g], pi[o * G + g]);
  __shared__ double sf[128];
  __shared__ long long si[128];
  sf[threadIdx.x] = f;
  si[threadIdx.x] = i;
  __syncthreads();
  for (int w = blockDim.x / 2; w > 0; w >>= 1) {
    if (threadIdx.x < w) {
      double f1 = sf[threadIdx.x]; long long i1 = si[threadIdx.x];
      tree_combine(a.op, exact, f1, i1, sf[threadIdx.x + w], si[threadIdx.x + w]);
      sf[threadIdx.x] = f1; si[threadIdx.x] = i1;
    }
    __syncthreads();
  }
  if (threadIdx.x != 0) return;
  f = sf[0];
  i = si[0];
  if (dtype_is_float_d(a.out_dtype)) {
    double v = exact ? (double)i : f;
    if (a.op == AMC_RED_MEAN) v = v / (double)a.R;
    store_num(a.out, a.out_dtype, o, nfl(v));
  } else {
    store_num(a.out, a.out_dtype, o, nex(i));
  }
}

int launch_reduce(const ReduceArgs& a, cudaStream_t s, void* scratch, size_t scratch_bytes, size_t* scratch_need) {
  const int sms = num_sms();
  // decide: ordered (bit-exact) unless few outputs over a long axis
  bool tree = (a.R > 16384) && (a.O < (long long)sms * 64);
  int G = 0;
  if (tree) {
    long long want = ((long long)sms * 8 + a.O - 1) / (a.O > 0 ? a.O : 1);
    G = (int)(want < 1 ? 1 : want > 1024 ? 1024 : want);
    long long per = (a.R + G - 1) / G;
    if (per < 1024) G = (int)((a.R + 1023) / 1024);
    if (G < 1) G = 1;
  }
  size_t need = tree ? (size_t)a.O * G * (sizeof(double) + sizeof(long long)) : 0;
  if (scratch_need) *scratch_need = need;
  if (!s && !scratch) return AMC_OK;  // sizing query only
  if (a.O == 0) return AMC_OK;
  if (fault_injected("launch")) return fail(AMC_ERR_INJECTED, "reduce: injected launch failure (AMC_FAULT=launch)");
  if (tree) {
    if (scratch_bytes < need || !scratch) return fail(AMC_ERR_INVALID, "reduce: scratch too small");
    double* pf = (double*)scratch;
    long long* pi = (long long*)((char*)scratch + (size_t)a.O * G * sizeof(double));
    dim3 g1((unsigned)G, (unsigned)a.O);
    k_reduce_tree1<<<g1, 256, 0, s>>>(a, pf, pi, G);
    AMC_CUDA(cudaGetLastError());
    k_reduce_tree2<<<(unsigned)a.O, 128, 0, s>>>(a, pf, pi, G);
    AMC_CUDA(cudaGetLastError());
    return AMC_OK;
  }
  if (a.R == 0) {
    // empty reduction: neutral element (and mean of nothing = 0/0 as the reference)
  }
  // tile shape: outputs per CTA so that the grid covers the SMs twice, RC to
  // fit shared memory
  long long O = a.O;
  int OT = 256;
  while (OT > 1 && (O + OT - 1) / OT < (long long)sms * 2) OT >>= 1;
  int RC = (int)(a.R < 1 ? 1 : a.R);
  int maxRC = (int)((48 * 1024) / (8 * OT)) - 1;
  if (maxRC < 1) maxRC = 1;
  if (RC > maxRC) RC = maxRC;
  // thread->element mapping: outputs fastest when the first leaf moves less
  // along the innermost kept axis than along the innermost reduced axis.
  int ofast = 1;
  if (a.orank > 0 && a.rrank > 0) {
    long long so = a.leaf_o[0].strides[a.orank - 1], sr = a.leaf_r[0][a.rrank - 1];
    so = so < 0 ? -so : so;
    sr = sr < 0 ? -sr : sr;
    ofast = (sr == 1 && so != 1) ? 0 : 1;
    if (so == 0 && sr != 0) ofast = 0;
  } else if (a.orank == 0) {
    ofast = 0;
  }
  const bool sumlike = a.op == AMC_RED_SUM || a.op == AMC_RED_MEAN;
  const bool src_float = a.src_dtype == AMC_F32 || a.src_dtype == AMC_F64;
  // column fold: few outputs adjacent in memory, a program of closed form,
  // tiles that TMA can move (amc_colfold.cu); else the staged form below
  if (OT < 8 && ofast && a.orank == 1 && a.rrank == 1) {
    const int rc = launch_colfold(a, s);
    if (rc != AMC_ERR_UNSUPPORTED) return rc;
  }
  // staged form: few outputs, adjacent in memory, small program
  if (OT < 8 && ofast && a.orank == 1 && a.rrank == 1 && a.nleaf >= 1 && a.nleaf <= 2 && a.prog.max_depth <= 3 &&
      a.prog.n > 0) {
    bool adjacent = true;
    for (int l = 0; l < a.nleaf; ++l) {
      const long long so = a.leaf_o[l].strides[0];
      adjacent = adjacent && (so == 0 || so == 1 || so == -1);
    }
    if (adjacent) {
      const unsigned gs = (unsigned)((O + kStOT - 1) / kStOT);
      const int mode = a.prog.all_float ? 0 : prog_int_only(a) ? 1 : 2;
#define AMC_STAGED(F)                                                                           \
  do {                                                                                          \
    if (mode == 0) k_reduce_staged<F, 0><<<gs, 256, 0, s>>>(a);                                 \
    else if (mode == 1) k_reduce_staged<F, 1><<<gs, 256, 0, s>>>(a);                            \
    else k_reduce_staged<F, 2><<<gs, 256, 0, s>>>(a);                                           \
  } while (0)
      if (sumlike && src_float && a.out_dtype == AMC_F64) AMC_STAGED(1);
      else if (sumlike && a.src_dtype == AMC_F32 && a.out_dtype == AMC_F32) AMC_STAGED(4);
      else if (sumlike && src_float && a.out_dtype == AMC_F32) AMC_STAGED(2);
      else if (sumlike && !src_float && (a.out_dtype == AMC_S32 || a.out_dtype == AMC_S64)) AMC_STAGED(3);
      else AMC_STAGED(0);
#undef AMC_STAGED
      AMC_CUDA(cudaGetLastError());
      return AMC_OK;
    }
  }
  size_t sm = (size_t)OT * (RC + 1) * 8;
  unsigned grid = (unsigned)((O + OT - 1) / OT);
  if (sumlike && src_float && a.out_dtype == AMC_F64)
    k_reduce_seq<1><<<grid, 256, sm, s>>>(a, OT, RC, ofast);
  else if (sumlike && a.src_dtype == AMC_F32 && a.out_dtype == AMC_F32)
    k_reduce_seq<4><<<grid, 256, sm, s>>>(a, OT, RC, ofast);
  else if (sumlike && src_float && a.out_dtype == AMC_F32)
    k_reduce_seq<2><<<grid, 256, sm, s>>>(a, OT, RC, ofast);
  else if (sumlike && !src_float && (a.out_dtype == AMC_S32 || a.out_dtype == AMC_S64))
    k_reduce_seq<3><<<grid, 256, sm, s>>>(a, OT, RC, ofast);
  else
    k_reduce_seq<0><<<grid, 256, sm, s>>>(a, OT, RC, ofast);
  AMC_CUDA(cudaGetLastError());
  return AMC_OK;
}

// ------------------------------------------------------------------ pad (structural-ops.scm:449-507)
__global__ void k_pad(const __grid_constant__ PadArgs a) {
  long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  long long stride = (long long)gridDim.x * blockDim.x;
  for (; i < a.total; i += stride) {
    long long rem = i, off = 0;
    bool inb = true;
    for (int d = a.rank - 1; d >= 0; --d) {
      long long c = rem % a.oshape[d];
      rem /= a.oshape[d];
      long long dim = a.sshape[d], s = c - a.before[d];
      if (a.mode == AMC_PAD_CONSTANT) {
        if (s < 0 || s >= dim) inb = false;
      } else if (a.mode == AMC_PAD_EDGE) {
        s = s < 0 ? 0 : (s >= dim ? dim - 1 : s);
      } else {
        for (int guard = 0; guard < 64 && (s < 0 || s >= dim); ++guard) s = s < 0 ? (-1 - s) : (2 * dim - s - 1);
        if (s < 0 || s >= dim) s = 0;
      }
      off += s * a.sstrides[d];
    }
    if (inb) store_num(a.out, a.out_dtype, i, load_num(a.src, a.src_dtype, off));
    else store_num(a.out, a.out_dtype, i, nfl(a.value));
  }
}

int launch_pad(const PadArgs& a, cudaStream_t s) {
  if (!a.total) return AMC_OK;
  k_pad<<<grid_for(a.total, 256), 256, 0, s>>>(a);
  AMC_CUDA(cudaGetLastError());
  return AMC_OK;
}

// ------------------------------------------------------------------ im2col (structural-ops.scm:581-627)
__global__ void k_im2col(const __grid_constant__ Im2colArgs a) {
  long long rows = a.C * a.KH * a.KW, cols = a.OH * a.OW, total = a.N * rows * cols;
  long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  long long stride = (long long)gridDim.x * blockDim.x;
  for (; i < total; i += stride) {
    long long c = i % cols, r = (i / cols) % rows, n = i / (rows * cols);
    long long ch = r / (a.KH * a.KW), kh = (r / a.KW) % a.KH, kw = r % a.KW, oh = c / a.OW, ow = c % a.OW;
    long long ih = oh * a.SH + kh - a.PH, iw = ow * a.SW + kw - a.PW;
    if (ih >= 0 && ih < a.H && iw >= 0 && iw < a.W)
      store_num(a.out, a.out_dtype, i, load_num(a.src, a.src_dtype, n * a.sN + ch * a.sC + ih * a.sH + iw * a.sW));
    else
      store_num(a.out, a.out_dtype, i, nfl(0.0));
  }
}

int launch_im2col(const Im2colArgs& a, cudaStream_t s) {
  long long total = a.N * a.C * a.KH * a.KW * a.OH * a.OW;
  if (!total) return AMC_OK;
  k_im2col<<<grid_for(total, 256), 256, 0, s>>>(a);
  AMC_CUDA(cudaGetLastError());
  return AMC_OK;
}

// ------------------------------------------------------------------ col2im
// Gather form of the reference's scatter-add (realization.scm:1196-1268):
// output (n,c,h,w) receives col[(n), (c,kh,kw), (oh,ow)] for every window
// position covering it, added in ascending col-row order (kh, then kw), the
// order the reference's outer col-row loop visits them.
__global__ void k_col2im(const __grid_constant__ Col2imArgs a) {
  long long total = a.N * a.C * a.H * a.W;
  long long rows = a.C * a.KH * a.KW, cols = a.OH * a.OW;
  long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  long long stride = (long long)gridDim.x * blockDim.x;
  const bool fp = a.out_dtype == AMC_F32 || a.out_dtype == AMC_F64;
  for (; i < total; i += stride) {
    long long w = i % a.W, h = (i / a.W) % a.H, c = (i / (a.W * a.H)) % a.C, n = i / (a.W * a.H * a.C);
    Num acc = nfl(0.0);
    if (!fp) acc = nex(0);
    for (int kh = 0; kh < a.KH; ++kh) {
      long long th = h + a.PH - kh;
      if (th < 0 || th % a.SH) continue;
      long long oh = th / a.SH;
      if (oh >= a.OH) continue;
      for (int kw = 0; kw < a.KW; ++kw) {
        long long tw = w + a.PW - kw;
        if (tw < 0 || tw % a.SW) continue;
        long long ow = tw / a.SW;
        if (ow >= a.OW) continue;
        long long r = c * a.KH * a.KW + kh * a.KW + kw;
        Num v = load_num(a.col, a.col_dtype, n * rows * cols + r * cols + oh * a.OW + ow);
        acc = round_store(a.out_dtype, bin_op(AMC_OP_ADD, acc, v));
      }
    }
    store_num(a.out, a.out_dtype, i, acc);
  }
}

int launch_col2im(const Col2imArgs& a, cudaStream_t s) {
  long long total = a.N * a.C * a.H * a.W;
  if (!total) return AMC_OK;
  k_col2im<<<grid_for(total, 256), 256, 0, s>>>(a);
  AMC_CUDA(cudaGetLastError());
  return AMC_OK;
}

// ------------------------------------------------------------------ stack / concat routing
__global__ void k_route(const __grid_constant__ RouteArgs a) {
  long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  long long stride = (long long)gridDim.x * blockDim.x;
  for (; i < a.total; i += stride) {
    long long idx[AMC_MAX_RANK];
    long long rem = i;
    for (int d = a.rank - 1; d >= 0; --d) { idx[d] = rem % a.oshape[d]; rem /= a.oshape[d]; }
    int src = 0;
    long long off = 0;
    if (a.is_stack) {
      src = (int)idx[a.axis];
      const DLeaf& L = a.srcs[src];
      int k = 0;
      for (int d = 0; d < a.rank; ++d) if (d != a.axis) off += idx[d] * L.strides[k++];
    } else {
      long long pos = idx[a.axis];
      while (src < a.nsrc - 1 && pos >= a.extents[src]) pos -= a.extents[src++];
      idx[a.axis] = pos;
      const DLeaf& L = a.srcs[src];
      for (int d = 0; d < a.rank; ++d) off += idx[d] * L.strides[d];
    }
    store_num(a.out, a.out_dtype, i, load_num(a.srcs[src].ptr, a.srcs[src].dtype, off));
  }
}

int launch_route(const RouteArgs& a, cudaStream_t s) {
  if (!a.total) return AMC_OK;
  k_route<<<grid_for(a.total, 256), 256, 0, s>>>(a);
  AMC_CUDA(cudaGetLastError());
  return AMC_OK;
}

// ------------------------------------------------------------------ scan / fold over the batch axis
// One thread per element position p of the accumulator.  acc starts as
// init[p]; step i evaluates the step program with leaf 0 = acc and leaf 1 =
// x[i, p], and rounds the value to the accumulator's dtype, as the i-th map
// node of the per-element tree stores it.  A scan stores every accumulator
// (row i of the output), a fold only the last.
template <bool ALLF>
__global__ void __launch_bounds__(256) k_scan(const __grid_constant__ ScanArgs a) {
  long long p = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (; p < a.P; p += stride) {
    long long off[2] = {0, 0};
    long long rem = p;
    for (int d = a.rank - 1; d >= 0; --d) {
      long long s = a.shape[d];
      long long c = rem % s;
      rem /= s;
      off[0] += c * a.leaf[0].strides[d];
      off[1] += c * a.leaf[1].strides[d];
    }
    if (ALLF) {
      double acc = load_f(a.leaf[0].ptr, a.leaf[0].dtype, off[0]);
      for (long long i = 0; i < a.n; ++i, off[1] += a.xstep) {
        acc = round_f(a.acc_dtype, eval_prog_f<true>(a.prog, a.leaf, off, 0, acc));
        if (a.keep) store_num(a.out, a.out_dtype, i * a.P + p, nfl(acc));
      }
      if (!a.keep) store_num(a.out, a.out_dtype, p, nfl(acc));
    } else {
      Num acc = load_num(a.leaf[0].ptr, a.leaf[0].dtype, off[0]);
      for (long long i = 0; i < a.n; ++i, off[1] += a.xstep) {
        acc = round_store(a.acc_dtype, eval_prog<true>(a.prog, a.leaf, off, 0, acc));
        if (a.keep) store_num(a.out, a.out_dtype, i * a.P + p, acc);
      }
      if (!a.keep) store_num(a.out, a.out_dtype, p, acc);
    }
  }
}

int launch_scan(const ScanArgs& a, cudaStream_t s) {
  if (a.P == 0 || a.n == 0) return AMC_OK;
  if (fault_injected("launch")) return fail(AMC_ERR_INJECTED, "scan: injected launch failure (AMC_FAULT=launch)");
  if (a.prog.all_float) k_scan<true><<<grid_for(a.P, 256), 256, 0, s>>>(a);
  else k_scan<false><<<grid_for(a.P, 256), 256, 0, s>>>(a);
  AMC_CUDA(cudaGetLastError());
  return AMC_OK;
}

// ------------------------------------------------------------------ GEMM (double accumulation)
// Tiles of 64x64 outputs, 4x4 per thread, K staged through shared memory as
// doubles.  Each output accumulates a*b in ascending k from 0.0 with separate
// multiply and add roundings, the reference's loop exactly.
__device__ __forceinline__ void gemm_tile(const GemmArgs& a, long long m0, long long n0, int tx, int ty,
                                          double (&acc)[4][4]) {
  __shared__ double As[16][64 + 1];
  __shared__ double Bs[16][64 + 1];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.0;
  for (long long k0 = 0; k0 < a.K; k0 += 16) {
    for (int e = threadIdx.x; e < 16 * 64; e += 256) {
      int kk = e / 64, mm = e % 64;
      long long m = m0 + mm, k = k0 + kk;
      As[kk][mm] = (m < a.M && k < a.K) ? load_f(a.A, a.a_dtype, m * a.sa0 + k * a.sa1) : 0.0;
      long long n = n0 + mm;
      Bs[kk][mm] = (n < a.N && k < a.K) ? load_f(a.B, a.b_dtype, k * a.sb0 + n * a.sb1) : 0.0;
    }
    __syncthreads();
    int kmax = (int)((a.K - k0) < 16 ? (a.K - k0) : 16);
    for (int kk = 0; kk < kmax; ++kk) {
      double av[4], bv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) av[i] = As[kk][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) bv[j] = Bs[kk][tx * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = __dadd_rn(acc[i][j], __dmul_rn(av[i], bv[j]));
    }
    __syncthreads();
  }
}

__global__ void __launch_bounds__(256) k_gemm(const __grid_constant__ GemmArgs a) {
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  const long long m0 = (long long)blockIdx.y * 64, n0 = (long long)blockIdx.x * 64;
  double acc[4][4];
  gemm_tile(a, m0, n0, tx, ty, acc);
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      long long m = m0 + ty * 4 + i, n = n0 + tx * 4 + j;
      if (m < a.M && n < a.N) {
        double v = acc[i][j];
        if (a.alpha != 1.0) v = __dmul_rn(a.alpha, v);
        if (a.beta != 0.0) v = __dadd_rn(v, __dmul_rn(a.beta, load_f(a.C, a.c_dtype, m * a.N + n)));
        store_num(a.C, a.c_dtype, m * a.N + n, nfl(v));
      }
    }
}

// GEMM with an element-wise epilogue.  Output element (m, n) is element
// m*N + n of the map's contiguous output.  The map program's leaf `leaf` is
// the GEMM result: its loads yield the product rounded to the GEMM's dtype,
// the value a separate map launch would have read back from C, so the result
// is bit-identical to the two launches and C is neither written nor read.
__global__ void __launch_bounds__(256) k_gemm_epi(const __grid_constant__ GemmEpiArgs a) {
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  const long long m0 = (long long)blockIdx.y * 64, n0 = (long long)blockIdx.x * 64;
  double acc[4][4];
  gemm_tile(a.g, m0, n0, tx, ty, acc);
  const MapArgs& e = a.map;
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      long long m = m0 + ty * 4 + i, n = n0 + tx * 4 + j;
      if (m < a.g.M && n < a.g.N) {
        const double v = acc[i][j];
        const double gv = a.g.c_dtype == AMC_F32 ? (double)__double2float_rn(v) : v;
        const long long idx = m * a.g.N + n;
        long long off[kMaxLeaves];
        for (int l = 0; l < e.nleaf; ++l) off[l] = 0;
        long long rem = idx;
        for (int d = e.rank - 1; d >= 0; --d) {
          long long s = e.shape[d];
          long long c = rem % s;
          rem /= s;
          for (int l = 0; l < e.nleaf; ++l) off[l] += c * e.leaf[l].strides[d];
        }
        if (e.prog.all_float) store_num(e.out, e.out_dtype, idx, nfl(eval_prog_f<true>(e.prog, e.leaf, off, a.leaf, gv)));
        else store_num(e.out, e.out_dtype, idx, eval_prog<true>(e.prog, e.leaf, off, a.leaf, nfl(gv)));
      }
    }
}

int launch_gemm(const GemmArgs& a, cudaStream_t s) {
  if (a.M == 0 || a.N == 0) return AMC_OK;
  if (fault_injected("launch")) return fail(AMC_ERR_INJECTED, "gemm: injected launch failure (AMC_FAULT=launch)");
  dim3 g((unsigned)((a.N + 63) / 64), (unsigned)((a.M + 63) / 64));
  k_gemm<<<g, 256, 0, s>>>(a);
  AMC_CUDA(cudaGetLastError());
  return AMC_OK;
}

int launch_gemm_epi(const GemmEpiArgs& a, cudaStream_t s) {
  if (a.g.M == 0 || a.g.N == 0) return AMC_OK;
  if (a.map.total != a.g.M * a.g.N || a.leaf < 0 || a.leaf >= a.map.nleaf || a.g.alpha != 1.0 || a.g.beta != 0.0)
    return fail(AMC_ERR_INVALID, "gemm epilogue: map does not cover the product");
  if (fault_injected("launch")) return fail(AMC_ERR_INJECTED, "gemm: injected launch failure (AMC_FAULT=launch)");
  dim3 g((unsigned)((a.g.N + 63) / 64), (unsigned)((a.g.M + 63) / 64));
  k_gemm_epi<<<g, 256, 0, s>>>(a);
  AMC_CUDA(cudaGetLastError());
  return AMC_OK;
}

// ------------------------------------------------------------------ attention (reference order)
// One warp per query row.  Pass 1: each lane computes whole scores for its
// keys with the j-sum in ascending order, stores them rounded to the dtype in
// shared memory and tracks the unrounded row max.  Pass 2: e_k = exp(s_k - max)
// rounded to the dtype; Z summed in double.  Pass 3: each lane owns output
// columns and accumulates (e_k/Z)*V[k,p] in ascending k.
__global__ void __launch_bounds__(128) k_attention_generic(const __grid_constant__ AttnArgs a) {
  extern __shared__ double att_sm[];
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32, wpb = blockDim.x / 32;
  double* s = att_sm + (size_t)warp * a.n;
  long long row = (long long)blockIdx.x * wpb + warp;
  long long rows = a.blocks * a.n;
  if (row >= rows) return;
  long long b = row / a.n, i = row % a.n;
  const long long qb = b * a.qb + i * a.q0, kb = b * a.kb, vb = b * a.vb;
  double rmax = -INFINITY;
  for (int k = lane; k < a.n; k += 32) {
    double acc = 0.0;
    for (int j = 0; j < a.dk; ++j)
      acc = __dadd_rn(acc, __dmul_rn(load_f(a.Q, a.dtype, qb + j * a.q1), load_f(a.K, a.dtype, kb + k * a.k0 + j * a.k1)));
    double score = __dmul_rn(a.scale, acc);
    s[k] = a.dtype == AMC_F32 ? (double)__double2float_rn(score) : score;
    rmax = score > rmax ? score : rmax;
  }
  for (int o = 16; o > 0; o >>= 1) {
    double t = __shfl_xor_sync(0xffffffffu, rmax, o);
    rmax = t > rmax ? t : rmax;
  }
  double Z = 0.0;
  for (int k = lane; k < a.n; k += 32) {
    double e = exp(s[k] - rmax);
    e = a.dtype == AMC_F32 ? (double)__double2float_rn(e) : e;
    s[k] = e;
    Z += e;
  }
  for (int o = 16; o > 0; o >>= 1) Z += __shfl_xor_sync(0xffffffffu, Z, o);
  __syncwarp();
  for (int p = lane; p < a.dv; p += 32) {
    double acc = 0.0;
    for (int k = 0; k < a.n; ++k)
      acc = __dadd_rn(acc, __dmul_rn(__ddiv_rn(s[k], Z), load_f(a.V, a.dtype, vb + k * a.v0 + p * a.v1)));
    store_num(a.O, a.dtype, row * a.dv + p, nfl(acc));
  }
}

int launch_attention_generic(const AttnArgs& a, cudaStream_t s) {
  long long rows = a.blocks * a.n;
  if (!rows) return AMC_OK;
  int wpb = 4;
  size_t sm = (size_t)wpb * a.n * sizeof(double);
  if (sm > 200 * 1024) {
    wpb = 1;
    sm = (size_t)a.n * sizeof(double);
  }
  if (sm > 200 * 1024) return fail(AMC_ERR_UNSUPPORTED, "attention: sequence too long for the reference-order kernel");
  if (sm > 48 * 1024) AMC_CUDA(cudaFuncSetAttribute(k_attention_generic, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm));
  k_attention_generic<<<(unsigned)((rows + wpb - 1) / wpb), wpb * 32, sm, s>>>(a);
  AMC_CUDA(cudaGetLastError());
  return AMC_OK;
}

}  // namespace amc
