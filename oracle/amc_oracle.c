/*
 * amc_oracle.c — CPU restatement of the reference's realization loops.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker for libamcuda: only the
 * tests, __graft_entry__.smoke() and bench.py's CPU-baseline / reference arm
 * load it.  The product path never links or calls it.
 *
 * The reference (iraikov/array-morphisms) is CHICKEN Scheme, and no CHICKEN
 * toolchain exists on this machine or the GPU machines, so the reference
 * itself cannot run here.  Each function below restates one loop of the
 * reference, cited by file:line, keeping its element order, its accumulation
 * order and its store conversions (typed-vector-set!, core.scm:649-658):
 *   - element-wise nodes compute in Scheme numbers (exact integers or IEEE
 *     doubles) and round only when the node is stored;
 *   - reductions accumulate sequentially in the source's logical row-major
 *     order INTO the typed output vector, so f32 partial sums are rounded to
 *     f32 at every step (realization.scm:1309-1388);
 *   - GEMM accumulates in double from 0.0 (blas-exec.scm:405-458).
 * The oracle is pinned against the reference tests' known answers (see
 * tests/golden/).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "../include/amc.h"

typedef struct orc_view {
  void*   data;
  int32_t dtype;
  int32_t rank;
  int64_t shape[AMC_MAX_RANK];
  int64_t strides[AMC_MAX_RANK];
  int64_t offset;
} orc_view;

/* ------------------------------------------------------------------ numbers
 * A Scheme number as the reference's loops see it: exact integer or flonum. */
typedef struct { int exact; int64_t i; double f; } num;

static num nx(int64_t i) { num r; r.exact = 1; r.i = i; r.f = (double)i; return r; }
static num nf(double f) { num r; r.exact = 0; r.i = 0; r.f = f; return r; }
static double fl(num a) { return a.exact ? (double)a.i : a.f; }

static int is_float_dtype(int32_t d) { return d == AMC_F32 || d == AMC_F64; }

/* typed-vector-ref (core.scm:638-647) */
static num tv_ref(const void* v, int32_t dtype, int64_t i) {
  switch (dtype) {
    case AMC_F32: return nf((double)((const float*)v)[i]);
    case AMC_F64: return nf(((const double*)v)[i]);
    case AMC_S32: return nx(((const int32_t*)v)[i]);
    case AMC_S64: return nx(((const int64_t*)v)[i]);
    case AMC_U32: return nx((int64_t)((const uint32_t*)v)[i]);
    case AMC_U64: return nx((int64_t)((const uint64_t*)v)[i]);
  }
  return nf(NAN);
}

/* typed-vector-set! (core.scm:649-658): f32/f64 store exact->inexact; integer
 * stores truncate toward zero; unsigned stores take abs of the truncation. */
static void tv_set(void* v, int32_t dtype, int64_t i, num x) {
  switch (dtype) {
    case AMC_F32: ((float*)v)[i] = (float)fl(x); break;
    case AMC_F64: ((double*)v)[i] = fl(x); break;
    case AMC_S32: ((int32_t*)v)[i] = (int32_t)(x.exact ? x.i : (int64_t)trunc(x.f)); break;
    case AMC_S64: ((int64_t*)v)[i] = x.exact ? x.i : (int64_t)trunc(x.f); break;
    case AMC_U32: { int64_t t = x.exact ? x.i : (int64_t)trunc(x.f); ((uint32_t*)v)[i] = (uint32_t)(t < 0 ? -t : t); } break;
    case AMC_U64: { int64_t t = x.exact ? x.i : (int64_t)trunc(x.f); ((uint64_t*)v)[i] = (uint64_t)(t < 0 ? -t : t); } break;
  }
}

/* the store conversion applied to a value without a vector (for CVT) */
static num store_round(int32_t dtype, num x) {
  switch (dtype) {
    case AMC_F32: return nf((double)(float)fl(x));
    case AMC_F64: return nf(fl(x));
    case AMC_S32: return nx((int32_t)(x.exact ? x.i : (int64_t)trunc(x.f)));
    case AMC_S64: return nx(x.exact ? x.i : (int64_t)trunc(x.f));
    case AMC_U32: { int64_t t = x.exact ? x.i : (int64_t)trunc(x.f); return nx((uint32_t)(t < 0 ? -t : t)); }
    case AMC_U64: { int64_t t = x.exact ? x.i : (int64_t)trunc(x.f); return nx(t < 0 ? -t : t); }
  }
  return x;
}

/* linear-to-multi-index (core.scm:458-474) */
static void unravel(int64_t lin, int32_t rank, const int64_t* shape, int64_t* idx) {
  for (int32_t d = rank - 1; d >= 0; --d) {
    int64_t s = shape[d];
    idx[d] = s ? lin % s : 0;
    lin = s ? lin / s : 0;
  }
}

static int64_t numel(int32_t rank, const int64_t* shape) {
  int64_t n = 1;
  for (int32_t d = 0; d < rank; ++d) n *= shape[d];
  return n;
}

/* retrieve-value (realization.scm:1465-1487): offset + sum idx*stride */
static int64_t phys(const orc_view* v, const int64_t* idx) {
  int64_t p = v->offset;
  for (int32_t d = 0; d < v->rank; ++d) p += idx[d] * v->strides[d];
  return p;
}

/* ------------------------------------------------------------------ combiners
 * get-binary-combiner (basic-ops.scm:125-133), get-unary-transformer
 * (:258-284), get-comparison-function (:427-435) with Scheme's exactness
 * contagion: exact op exact stays exact (division of exact integers that
 * does not divide evenly is a rational, represented here by its double). */
static int64_t ipow(int64_t a, int64_t b) {
  int64_t r = 1;
  while (b > 0) { if (b & 1) r *= a; a *= a; b >>= 1; }
  return r;
}

static int apply_unary(int op, num a, num* out) {
  double x = fl(a);
  switch (op) {
    case AMC_OP_NEG: *out = a.exact ? nx(-a.i) : nf(-a.f); return 0;
    case AMC_OP_ABS: *out = a.exact ? nx(a.i < 0 ? -a.i : a.i) : nf(fabs(a.f)); return 0;
    case AMC_OP_FLOOR: *out = a.exact ? a : nf(floor(a.f)); return 0;
    case AMC_OP_CEIL: *out = a.exact ? a : nf(ceil(a.f)); return 0;
    case AMC_OP_SQRT:
      if (a.exact && a.i >= 0) {
        int64_t r = (int64_t)llround(sqrt((double)a.i));
        if (r * r == a.i) { *out = nx(r); return 0; }
      }
      *out = nf(sqrt(x)); return 0;
    case AMC_OP_EXP: *out = nf(exp(x)); return 0;
    case AMC_OP_LOG: *out = nf(log(x)); return 0;
    case AMC_OP_SIN: *out = nf(sin(x)); return 0;
    case AMC_OP_COS: *out = nf(cos(x)); return 0;
    case AMC_OP_TAN: *out = nf(tan(x)); return 0;
    case AMC_OP_RELU: *out = nf(x > 0.0 ? x : 0.0); return 0;
    case AMC_OP_SIGMOID: *out = nf(1.0 / (1.0 + exp(-x))); return 0;
    case AMC_OP_TANH: { double e2 = exp(2.0 * x); *out = nf((e2 - 1.0) / (e2 + 1.0)); return 0; }
  }
  return -1;
}

static int apply_binary(int op, num a, num b, num* out) {
  int ex = a.exact && b.exact;
  double x = fl(a), y = fl(b);
  switch (op) {
    case AMC_OP_ADD: *out = ex ? nx(a.i + b.i) : nf(x + y); return 0;
    case AMC_OP_SUB: *out = ex ? nx(a.i - b.i) : nf(x - y); return 0;
    case AMC_OP_MUL: *out = ex ? nx(a.i * b.i) : nf(x * y); return 0;
    case AMC_OP_DIV:
      if (ex) {
        if (b.i == 0) return -2;  /* Scheme: division by zero error */
        if (a.i % b.i == 0) { *out = nx(a.i / b.i); return 0; }
        *out = nf((double)a.i / (double)b.i); return 0;
      }
      *out = nf(x / y); return 0;
    case AMC_OP_POW:
      if (ex && b.i >= 0) { *out = nx(ipow(a.i, b.i)); return 0; }
      *out = nf(pow(x, y)); return 0;
    case AMC_OP_MAX: *out = ex ? nx(a.i > b.i ? a.i : b.i) : nf(x > y ? x : y); return 0;
    case AMC_OP_MIN: *out = ex ? nx(a.i < b.i ? a.i : b.i) : nf(x < y ? x : y); return 0;
    case AMC_OP_GT: *out = nf(ex ? (a.i > b.i) : (x > y)); return 0;
    case AMC_OP_LT: *out = nf(ex ? (a.i < b.i) : (x < y)); return 0;
    case AMC_OP_EQ: *out = nf(ex ? (a.i == b.i) : (x == y)); return 0;
    case AMC_OP_GE: *out = nf(ex ? (a.i >= b.i) : (x >= y)); return 0;
    case AMC_OP_LE: *out = nf(ex ? (a.i <= b.i) : (x <= y)); return 0;
  }
  return -1;
}

static int run_prog(const amc_insn* prog, int32_t plen, const num* in, num* out) {
  num st[AMC_STACK_MAX];
  int sp = 0;
  for (int32_t pc = 0; pc < plen; ++pc) {
    const amc_insn* I = &prog[pc];
    if (I->op == AMC_OP_LOAD) { if (sp >= AMC_STACK_MAX) return -3; st[sp++] = in[I->a]; continue; }
    if (I->op == AMC_OP_CONST) { if (sp >= AMC_STACK_MAX) return -3; st[sp++] = nf(I->imm); continue; }
    if (I->op == AMC_OP_ICONST) { if (sp >= AMC_STACK_MAX) return -3; st[sp++] = nx((int64_t)I->imm); continue; }
    if (I->op == AMC_OP_CVT) { if (sp < 1) return -3; st[sp - 1] = store_round(I->a, st[sp - 1]); continue; }
    if (I->op >= AMC_OP_NEG && I->op <= AMC_OP_TANH) {
      if (sp < 1) return -3;
      int rc = apply_unary(I->op, st[sp - 1], &st[sp - 1]);
      if (rc) return rc;
      continue;
    }
    if (sp < 2) return -3;
    int rc = apply_binary(I->op, st[sp - 2], st[sp - 1], &st[sp - 2]);
    if (rc) return rc;
    --sp;
  }
  if (sp != 1) return -3;
  *out = st[0];
  return 0;
}

/* ------------------------------------------------------------------ compute node
 * execute-compute-morphism (realization.scm:876-933) and its flat fast paths
 * (:935-977), which visit the same elements in the same order: for every
 * output element in row-major order, read each operand through its
 * broadcast index function (basic-ops.scm:100-115, here a view with stride
 * 0 on broadcast axes, built by the caller), apply the combiner, store. */
int orc_map(void* out, int32_t out_dtype, int32_t rank, const int64_t* shape,
            int32_t n_ops, const orc_view* ops, const amc_insn* prog, int32_t plen) {
  int64_t n = numel(rank, shape), idx[AMC_MAX_RANK];
  num in[8];
  if (n_ops > 8) return -1;
  for (int64_t i = 0; i < n; ++i) {
    unravel(i, rank, shape, idx);
    for (int32_t k = 0; k < n_ops; ++k) {
      const orc_view* v = &ops[k];
      /* broadcast: operand rank may be lower; align trailing axes */
      int64_t p = v->offset;
      int32_t lead = rank - v->rank;
      for (int32_t d = 0; d < v->rank; ++d) p += (v->shape[d] == 1 ? 0 : idx[lead + d]) * v->strides[d];
      in[k] = tv_ref(v->data, v->dtype, p);
    }
    num r;
    int rc = run_prog(prog, plen, in, &r);
    if (rc) return rc;
    tv_set(out, out_dtype, i, r);
  }
  return 0;
}

/* ------------------------------------------------------------------ reduction
 * execute-reduction-morphism (realization.scm:1309-1388).  Output initialised
 * with the op's neutral element through typed-vector-set!; integer max/min
 * would store +-inf into an integer vector, an error in the reference. */
int orc_reduce(void* out, int32_t out_dtype, const orc_view* src, int64_t axes_mask,
               int32_t keepdims, int32_t op) {
  int64_t out_shape[AMC_MAX_RANK];
  int32_t out_rank = 0;
  int64_t reduce_size = 1;
  for (int32_t d = 0; d < src->rank; ++d) {
    if (axes_mask & (1LL << d)) { reduce_size *= src->shape[d]; if (keepdims) out_shape[out_rank++] = 1; }
    else out_shape[out_rank++] = src->shape[d];
  }
  int64_t out_n = numel(out_rank, out_shape);
  if (!is_float_dtype(out_dtype) && (op == AMC_RED_MAX || op == AMC_RED_MIN)) return -4;
  num init = (op == AMC_RED_PROD) ? nf(1.0) : (op == AMC_RED_MAX) ? nf(-INFINITY)
           : (op == AMC_RED_MIN) ? nf(INFINITY) : nf(0.0);
  for (int64_t i = 0; i < out_n; ++i) tv_set(out, out_dtype, i, init);

  int64_t src_n = numel(src->rank, src->shape), idx[AMC_MAX_RANK];
  int64_t ostr[AMC_MAX_RANK];
  {  /* compute-strides of the output shape */
    int64_t s = 1;
    for (int32_t d = out_rank - 1; d >= 0; --d) { ostr[d] = s; s *= out_shape[d]; }
  }
  int binop = op == AMC_RED_PROD ? AMC_OP_MUL : op == AMC_RED_MAX ? AMC_OP_MAX
            : op == AMC_RED_MIN ? AMC_OP_MIN : AMC_OP_ADD;
  for (int64_t i = 0; i < src_n; ++i) {
    unravel(i, src->rank, src->shape, idx);
    int64_t p = phys(src, idx);
    int64_t o = 0;
    int32_t od = 0;
    for (int32_t d = 0; d < src->rank; ++d) {
      if (axes_mask & (1LL << d)) { if (keepdims) ++od; }
      else { o += idx[d] * ostr[od]; ++od; }
    }
    num a = tv_ref(out, out_dtype, o), b = tv_ref(src->data, src->dtype, p), r;
    apply_binary(binop, a, b, &r);
    tv_set(out, out_dtype, o, r);
  }
  if (op == AMC_RED_MEAN) {
    for (int64_t i = 0; i < out_n; ++i) {
      num v = tv_ref(out, out_dtype, i), r;
      apply_binary(AMC_OP_DIV, v, nx(reduce_size), &r);
      tv_set(out, out_dtype, i, r);
    }
  }
  return 0;
}

/* ------------------------------------------------------------------ copies
 * execute-affine-morphism, identity branch (realization.scm:849-862): output
 * element i takes the source's i-th element in the source's logical
 * row-major order (a reshape of a non-contiguous view). */
int orc_copy_logical(void* out, int32_t out_dtype, const orc_view* src) {
  int64_t n = numel(src->rank, src->shape), idx[AMC_MAX_RANK];
  for (int64_t i = 0; i < n; ++i) {
    unravel(i, src->rank, src->shape, idx);
    tv_set(out, out_dtype, i, tv_ref(src->data, src->dtype, phys(src, idx)));
  }
  return 0;
}

/* make-pad-index-fn (structural-ops.scm:449-507) run by
 * execute-procedure-index-fn (realization.scm:1425-1459). */
int orc_pad(void* out, int32_t out_dtype, int32_t rank, const int64_t* out_shape,
            const orc_view* src, const int64_t* pads, int32_t mode, double value) {
  int64_t n = numel(rank, out_shape), idx[AMC_MAX_RANK], sidx[AMC_MAX_RANK];
  for (int64_t i = 0; i < n; ++i) {
    unravel(i, rank, out_shape, idx);
    int inb = 1;
    for (int32_t d = 0; d < rank; ++d) {
      int64_t dim = src->shape[d], s = idx[d] - pads[2 * d];
      if (mode == AMC_PAD_CONSTANT) {
        if (s < 0 || s >= dim) inb = 0;
      } else if (mode == AMC_PAD_EDGE) {
        s = s < 0 ? 0 : (s >= dim ? dim - 1 : s);
      } else {
        /* reflect: -1-idx below, 2*dim-idx-1 above, repeated */
        while (s < 0 || s >= dim) s = (s < 0) ? (-1 - s) : (2 * dim - s - 1);
      }
      sidx[d] = s;
    }
    if (!inb) tv_set(out, out_dtype, i, nf(value));
    else tv_set(out, out_dtype, i, tv_ref(src->data, src->dtype, phys(src, sidx)));
  }
  return 0;
}

/* make-im2col-index-fn (structural-ops.scm:581-627): row = c*KH*KW + kh*KW + kw,
 * col = oh*OW + ow, in-bounds -> x[(n), c, oh*SH+kh-PH, ow*SW+kw-PW] else 0. */
int orc_im2col(void* out, int32_t out_dtype, const orc_view* src, int32_t batched,
               int32_t KH, int32_t KW, int32_t SH, int32_t SW, int32_t PH, int32_t PW) {
  int32_t b = batched ? 1 : 0;
  int64_t N = batched ? src->shape[0] : 1, C = src->shape[b], H = src->shape[b + 1], W = src->shape[b + 2];
  int64_t OH = 1 + (H + 2 * PH - KH) / SH, OW = 1 + (W + 2 * PW - KW) / SW;
  int64_t rows = C * KH * KW, cols = OH * OW, i = 0, sidx[4];
  for (int64_t n = 0; n < N; ++n)
    for (int64_t r = 0; r < rows; ++r)
      for (int64_t c = 0; c < cols; ++c, ++i) {
        int64_t ch = r / (KH * KW), kh = (r / KW) % KH, kw = r % KW, oh = c / OW, ow = c % OW;
        int64_t ih = oh * SH + kh - PH, iw = ow * SW + kw - PW;
        if (ih >= 0 && ih < H && iw >= 0 && iw < W) {
          int32_t k = 0;
          if (batched) sidx[k++] = n;
          sidx[k++] = ch; sidx[k++] = ih; sidx[k++] = iw;
          tv_set(out, out_dtype, i, tv_ref(src->data, src->dtype, phys(src, sidx)));
        } else {
          tv_set(out, out_dtype, i, nf(0.0));
        }
      }
  return 0;
}

/* execute-col2im-unbatched / -batched (realization.scm:1123-1268): zero the
 * image, then for col-row (outer) and col-col (inner) add col into the image
 * where the window position is in bounds.  The reference addresses the col
 * data linearly from index 0 (it ignores the operand's strides), so the
 * caller passes a contiguous col. */
int orc_col2im(void* out, int32_t dtype, int32_t batched, int64_t N, int64_t C, int64_t H, int64_t W,
               const void* col, int32_t col_dtype,
               int32_t KH, int32_t KW, int32_t SH, int32_t SW, int32_t PH, int32_t PW) {
  int64_t OH = 1 + (H + 2 * PH - KH) / SH, OW = 1 + (W + 2 * PW - KW) / SW;
  int64_t rows = C * KH * KW, cols = OH * OW, total = (batched ? N : 1) * C * H * W;
  for (int64_t i = 0; i < total; ++i) tv_set(out, dtype, i, nf(0.0));
  int64_t nb = batched ? N : 1;
  for (int64_t n = 0; n < nb; ++n)
    for (int64_t r = 0; r < rows; ++r) {
      int64_t c = r / (KH * KW), kh = (r / KW) % KH, kw = r % KW;
      for (int64_t cc = 0; cc < cols; ++cc) {
        int64_t oh = cc / OW, ow = cc % OW, h = oh * SH + kh - PH, w = ow * SW + kw - PW;
        if (h >= 0 && h < H && w >= 0 && w < W) {
          int64_t o = ((n * C + c) * H + h) * W + w;
          num a = tv_ref(out, dtype, o), v = tv_ref(col, col_dtype, n * rows * cols + r * cols + cc), s;
          apply_binary(AMC_OP_ADD, a, v, &s);
          tv_set(out, dtype, o, s);
        }
      }
    }
  return 0;
}

/* execute-routing-morphism with the stack / concat index functions
 * (realization.scm:1046-1081, index-functions.scm:375-410). */
int orc_route(void* out, int32_t out_dtype, int32_t rank, const int64_t* out_shape,
              int32_t n_ops, const orc_view* ops, int32_t axis, int32_t is_stack) {
  int64_t n = numel(rank, out_shape), idx[AMC_MAX_RANK], sidx[AMC_MAX_RANK];
  for (int64_t i = 0; i < n; ++i) {
    unravel(i, rank, out_shape, idx);
    int32_t src = 0;
    if (is_stack) {
      src = (int32_t)idx[axis];
      int32_t k = 0;
      for (int32_t d = 0; d < rank; ++d) if (d != axis) sidx[k++] = idx[d];
    } else {
      int64_t pos = idx[axis];
      while (src < n_ops - 1 && pos >= ops[src].shape[axis]) pos -= ops[src++].shape[axis];
      for (int32_t d = 0; d < rank; ++d) sidx[d] = idx[d];
      sidx[axis] = pos;
    }
    tv_set(out, out_dtype, i, tv_ref(ops[src].data, ops[src].dtype, phys(&ops[src], sidx)));
  }
  return 0;
}

/* ------------------------------------------------------------------ BLAS
 * execute-scheme-gemm (blas-exec.scm:405-458): stride-aware triple loop,
 * accumulator starts at 0.0 (inexact) and adds a*b in k order. */
int orc_gemm(void* out, int32_t out_dtype, const orc_view* A, const orc_view* B) {
  int64_t M = A->shape[0], K = A->shape[1], N = B->shape[1];
  for (int64_t i = 0; i < M; ++i)
    for (int64_t j = 0; j < N; ++j) {
      num acc = nf(0.0), t;
      for (int64_t k = 0; k < K; ++k) {
        num a = tv_ref(A->data, A->dtype, A->offset + i * A->strides[0] + k * A->strides[1]);
        num b = tv_ref(B->data, B->dtype, B->offset + k * B->strides[0] + j * B->strides[1]);
        apply_binary(AMC_OP_MUL, a, b, &t);
        apply_binary(AMC_OP_ADD, acc, t, &acc);
      }
      tv_set(out, out_dtype, i * N + j, acc);
    }
  return 0;
}

/* execute-scheme-gemv (blas-exec.scm:460-500) and -dot (:502-530). */
int orc_gemv(void* out, int32_t out_dtype, const orc_view* A, const orc_view* x) {
  int64_t M = A->shape[0], N = A->shape[1];
  for (int64_t i = 0; i < M; ++i) {
    num acc = nf(0.0), t;
    for (int64_t j = 0; j < N; ++j) {
      num a = tv_ref(A->data, A->dtype, A->offset + i * A->strides[0] + j * A->strides[1]);
      num b = tv_ref(x->data, x->dtype, x->offset + j * x->strides[0]);
      apply_binary(AMC_OP_MUL, a, b, &t);
      apply_binary(AMC_OP_ADD, acc, t, &acc);
    }
    tv_set(out, out_dtype, i, acc);
  }
  return 0;
}

int orc_dot(void* out, int32_t out_dtype, const orc_view* x, const orc_view* y) {
  num acc = nf(0.0), t;
  for (int64_t j = 0; j < x->shape[0]; ++j) {
    num a = tv_ref(x->data, x->dtype, x->offset + j * x->strides[0]);
    num b = tv_ref(y->data, y->dtype, y->offset + j * y->strides[0]);
    apply_binary(AMC_OP_MUL, a, b, &t);
    apply_binary(AMC_OP_ADD, acc, t, &acc);
  }
  tv_set(out, out_dtype, 0, acc);
  return 0;
}

/* ------------------------------------------------------------------ conv
 * execute-conv2d-blas (realization.scm:166-252): per image, im2col into a
 * contiguous (C*KH*KW, OH*OW) slab, then GEMM of the flattened weight
 * (C_out, C*KH*KW) with it; results copied to the NCHW output. */
int orc_conv2d(void* out, int32_t dtype, const orc_view* X, const orc_view* Wt, int32_t batched,
               int32_t KH, int32_t KW, int32_t SH, int32_t SW, int32_t PH, int32_t PW) {
  int32_t b = batched ? 1 : 0;
  int64_t N = batched ? X->shape[0] : 1, C = X->shape[b], H = X->shape[b + 1], W = X->shape[b + 2];
  int64_t OH = 1 + (H + 2 * PH - KH) / SH, OW = 1 + (W + 2 * PW - KW) / SW;
  int64_t KK = C * KH * KW, OO = OH * OW, CO = Wt->shape[0];
  size_t esz = dtype == AMC_F32 ? 4 : 8;
  void* col = malloc((size_t)(KK * OO) * esz);
  void* g = malloc((size_t)(CO * OO) * esz);
  if (!col || !g) { free(col); free(g); return -5; }
  orc_view w2 = *Wt;  /* weight reshaped to (C_out, KK): contiguous */
  w2.rank = 2; w2.shape[0] = CO; w2.shape[1] = KK; w2.strides[0] = KK; w2.strides[1] = 1;
  for (int64_t n = 0; n < N; ++n) {
    orc_view xi = *X;
    if (batched) {  /* sample n as a (C,H,W) view */
      xi.offset = X->offset + n * X->strides[0];
      xi.rank = 3;
      for (int d = 0; d < 3; ++d) { xi.shape[d] = X->shape[d + 1]; xi.strides[d] = X->strides[d + 1]; }
    }
    orc_im2col(col, dtype, &xi, 0, KH, KW, SH, SW, PH, PW);
    orc_view cv; memset(&cv, 0, sizeof cv);
    cv.data = col; cv.dtype = dtype; cv.rank = 2; cv.shape[0] = KK; cv.shape[1] = OO; cv.strides[0] = OO; cv.strides[1] = 1;
    orc_gemm(g, dtype, &w2, &cv);
    memcpy((char*)out + (size_t)(n * CO * OO) * esz, g, (size_t)(CO * OO) * esz);
  }
  free(col); free(g);
  return 0;
}

/* ------------------------------------------------------------------ attention
 * %attn-2d! (realization.scm:279-326) over the leading blocks
 * (execute-fused-attention, :328-396).  Scores and exponentials are stored
 * into dtype-typed scratch vectors (rounded for f32); Z and the output
 * accumulator are doubles; the output is stored as dtype. */
int orc_attention(void* out, int32_t dtype, const orc_view* Q, const orc_view* K, const orc_view* V,
                  int32_t n_leading, double scale) {
  int32_t qr = Q->rank, vr = V->rank;
  int64_t n = Q->shape[qr - 2], dk = Q->shape[qr - 1], dv = V->shape[vr - 1];
  int64_t nb = 1;
  for (int32_t i = 0; i < n_leading; ++i) nb *= Q->shape[i];
  int64_t qr0 = Q->strides[qr - 2], qr1 = Q->strides[qr - 1];
  int64_t kr0 = K->strides[qr - 2], kr1 = K->strides[qr - 1];
  int64_t vr0 = V->strides[vr - 2], vr1 = V->strides[vr - 1];
  int64_t qb = n_leading ? Q->strides[qr - 3] : 0, kb = n_leading ? K->strides[qr - 3] : 0,
          vb = n_leading ? V->strides[vr - 3] : 0;
  size_t esz = dtype == AMC_F32 ? 4 : 8;
  void* s = malloc((size_t)n * esz);
  void* e = malloc((size_t)n * esz);
  if (!s || !e) { free(s); free(e); return -5; }
  for (int64_t b = 0; b < nb; ++b) {
    int64_t q0 = Q->offset + b * qb, k0 = K->offset + b * kb, v0 = V->offset + b * vb, o0 = b * n * dv;
    for (int64_t i = 0; i < n; ++i) {
      double rmax = -INFINITY;
      for (int64_t k = 0; k < n; ++k) {
        double acc = 0.0;
        for (int64_t j = 0; j < dk; ++j)
          acc += fl(tv_ref(Q->data, Q->dtype, q0 + i * qr0 + j * qr1)) *
                 fl(tv_ref(K->data, K->dtype, k0 + k * kr0 + j * kr1));
        double score = scale * acc;
        tv_set(s, dtype, k, nf(score));
        if (score > rmax) rmax = score;  /* the unrounded score, as :307 */
      }
      double Z = 0.0;
      for (int64_t k = 0; k < n; ++k) {
        double ek = exp(fl(tv_ref(s, dtype, k)) - rmax);
        tv_set(e, dtype, k, nf(ek));
        Z += ek;
      }
      for (int64_t p = 0; p < dv; ++p) {
        double acc = 0.0;
        for (int64_t k = 0; k < n; ++k)
          acc += (fl(tv_ref(e, dtype, k)) / Z) * fl(tv_ref(V->data, V->dtype, v0 + k * vr0 + p * vr1));
        tv_set(out, dtype, o0 + i * dv + p, nf(acc));
      }
    }
  }
  free(s); free(e);
  return 0;
}

/* Attention backward has no reference implementation (grad.scm and ssa-vjp
 * have no attention rule).  This is the standard softmax-attention VJP in
 * double precision, used as the oracle for dQ, dK, dV:
 *   P = softmax(scale Q K^T), O = P V,
 *   dV = P^T dO, dP = dO V^T, dS = P * (dP - rowsum(dO * O)), dQ = scale dS K,
 *   dK = scale dS^T Q.  Contiguous (B, n, d) blocks. */
int orc_attention_bwd(const float* Q, const float* K, const float* V, const float* dO,
                      float* dQ, float* dK, float* dV, int64_t nb, int64_t n, int64_t dk, int64_t dv,
                      double scale) {
  double* P = (double*)malloc((size_t)(n * n) * sizeof(double));
  double* O = (double*)malloc((size_t)(n * dv) * sizeof(double));
  double* dS = (double*)malloc((size_t)(n * n) * sizeof(double));
  if (!P || !O || !dS) { free(P); free(O); free(dS); return -5; }
  for (int64_t b = 0; b < nb; ++b) {
    const float *q = Q + b * n * dk, *k = K + b * n * dk, *v = V + b * n * dv, *g = dO + b * n * dv;
    float *gq = dQ + b * n * dk, *gk = dK + b * n * dk, *gv = dV + b * n * dv;
    for (int64_t i = 0; i < n; ++i) {
      double m = -INFINITY;
      for (int64_t j = 0; j < n; ++j) {
        double a = 0; for (int64_t c = 0; c < dk; ++c) a += (double)q[i * dk + c] * k[j * dk + c];
        P[i * n + j] = scale * a; if (P[i * n + j] > m) m = P[i * n + j];
      }
      double z = 0; for (int64_t j = 0; j < n; ++j) { P[i * n + j] = exp(P[i * n + j] - m); z += P[i * n + j]; }
      for (int64_t j = 0; j < n; ++j) P[i * n + j] /= z;
      for (int64_t p = 0; p < dv; ++p) { double a = 0; for (int64_t j = 0; j < n; ++j) a += P[i * n + j] * v[j * dv + p]; O[i * dv + p] = a; }
    }
    for (int64_t j = 0; j < n; ++j)
      for (int64_t p = 0; p < dv; ++p) { double a = 0; for (int64_t i = 0; i < n; ++i) a += P[i * n + j] * g[i * dv + p]; gv[j * dv + p] = (float)a; }
    for (int64_t i = 0; i < n; ++i) {
      double D = 0; for (int64_t p = 0; p < dv; ++p) D += (double)g[i * dv + p] * O[i * dv + p];
      for (int64_t j = 0; j < n; ++j) {
        double dp = 0; for (int64_t p = 0; p < dv; ++p) dp += (double)g[i * dv + p] * v[j * dv + p];
        dS[i * n + j] = P[i * n + j] * (dp - D);
      }
    }
    for (int64_t i = 0; i < n; ++i)
      for (int64_t c = 0; c < dk; ++c) { double a = 0; for (int64_t j = 0; j < n; ++j) a += dS[i * n + j] * k[j * dk + c]; gq[i * dk + c] = (float)(scale * a); }
    for (int64_t j = 0; j < n; ++j)
      for (int64_t c = 0; c < dk; ++c) { double a = 0; for (int64_t i = 0; i < n; ++i) a += dS[i * n + j] * q[i * dk + c]; gk[j * dk + c] = (float)(scale * a); }
  }
  free(P); free(O); free(dS);
  return 0;
}

/* ------------------------------------------------------------------ SSA linear regression step
 * The replayed SSA program of loss = mean((X w - y)^2) and its VJP
 * (ssa.scm:517-1033: matmul rule :916-933, mean rule :953-963, mul rule
 * :739-750), executed per step as the reference's kernels would:
 *   pred = X w (double accumulation over k), r = pred - y, loss = sum(r*r)/N,
 *   g = 1.0/N broadcast, dr = g*r + g*r, dw = X^T dr (accumulation over i),
 *   w -= lr * dw.  X is (N, D) row-major. */
int orc_linreg(const double* X, const double* y, double* w, int64_t N, int32_t D, int32_t steps,
               double lr, double* losses) {
  double* r = (double*)malloc((size_t)N * sizeof(double));
  double* dw = (double*)malloc((size_t)D * sizeof(double));
  if (!r || !dw) { free(r); free(dw); return -5; }
  for (int32_t s = 0; s < steps; ++s) {
    double loss = 0.0, g = 1.0 / (double)N;
    for (int64_t i = 0; i < N; ++i) {
      double acc = 0.0;
      for (int32_t k = 0; k < D; ++k) acc += X[i * D + k] * w[k];
      r[i] = acc - y[i];
      loss += r[i] * r[i];
    }
    loss = loss / (double)N;
    for (int32_t k = 0; k < D; ++k) dw[k] = 0.0;
    for (int64_t i = 0; i < N; ++i) {
      double dri = g * r[i] + g * r[i];
      for (int32_t k = 0; k < D; ++k) dw[k] += X[i * D + k] * dri;
    }
    for (int32_t k = 0; k < D; ++k) w[k] = w[k] - lr * dw[k];
    if (losses) losses[s] = loss;
  }
  free(r); free(dw);
  return 0;
}

/* ------------------------------------------------------------------ buffer colouring
 * compute-last-uses! (context.scm:282-295) then allocate-buffers
 * (context.scm:325-412): greedy by birth order, per dtype an active list
 * (newest first) and a free list (expired entries pushed on its front in
 * active-list order); the first free entry whose size is large enough is
 * reused, else a new buffer is made.  Pinned records live to the end. */
int orc_colour(int32_t n, const int32_t* dtypes, const int64_t* sizes, const int32_t* in_off,
               const int32_t* inputs, const int32_t* pinned, int32_t* assignment, int32_t* n_buffers) {
  int32_t* last = (int32_t*)malloc(sizeof(int32_t) * (size_t)(n > 0 ? n : 1));
  int32_t *act_id = (int32_t*)malloc(sizeof(int32_t) * (size_t)(n + 1)), *act_end = (int32_t*)malloc(sizeof(int32_t) * (size_t)(n + 1)),
          *act_dt = (int32_t*)malloc(sizeof(int32_t) * (size_t)(n + 1));
  int32_t *fr_id = (int32_t*)malloc(sizeof(int32_t) * (size_t)(n + 1)), *fr_dt = (int32_t*)malloc(sizeof(int32_t) * (size_t)(n + 1));
  int64_t* fr_sz = (int64_t*)malloc(sizeof(int64_t) * (size_t)(n + 1));
  int64_t* buf_sz = (int64_t*)malloc(sizeof(int64_t) * (size_t)(n + 1));
  int32_t na = 0, nf_ = 0, nb = 0;
  for (int32_t i = 0; i < n; ++i) last[i] = i;
  for (int32_t i = 0; i < n; ++i)
    for (int32_t k = in_off[i]; k < in_off[i + 1]; ++k) {
      int32_t p = inputs[k];
      if (p >= 0 && i > last[p]) last[p] = i;
    }
  for (int32_t i = 0; i < n; ++i) if (pinned && pinned[i]) last[i] = n - 1;
  for (int32_t i = 0; i < n; ++i) {
    int32_t dt = dtypes[i];
    /* active entries of this dtype, in list order (newest first) are stored
     * in act_* with index 0 = newest.  Expire those with end < i. */
    int32_t expired_ids[1024]; int32_t ne = 0;
    int32_t w = 0;
    for (int32_t a = 0; a < na; ++a) {
      if (act_dt[a] == dt && act_end[a] < i) { if (ne < 1024) expired_ids[ne++] = act_id[a]; }
      else { act_id[w] = act_id[a]; act_end[w] = act_end[a]; act_dt[w] = act_dt[a]; ++w; }
    }
    na = w;
    /* for-each over expired (list order) consing onto the dtype's free list:
     * the last expired ends up first. */
    for (int32_t e = 0; e < ne; ++e) {
      for (int32_t f = nf_; f > 0; --f) { fr_id[f] = fr_id[f - 1]; fr_sz[f] = fr_sz[f - 1]; fr_dt[f] = fr_dt[f - 1]; }
      fr_id[0] = expired_ids[e]; fr_sz[0] = buf_sz[expired_ids[e]]; fr_dt[0] = dt; ++nf_;
    }
    int32_t pick = -1;
    for (int32_t f = 0; f < nf_; ++f) if (fr_dt[f] == dt && fr_sz[f] >= sizes[i]) { pick = f; break; }
    int32_t bid;
    if (pick >= 0) {
      bid = fr_id[pick];
      if (sizes[i] > buf_sz[bid]) buf_sz[bid] = sizes[i];
      for (int32_t f = pick; f < nf_ - 1; ++f) { fr_id[f] = fr_id[f + 1]; fr_sz[f] = fr_sz[f + 1]; fr_dt[f] = fr_dt[f + 1]; }
      --nf_;
    } else {
      bid = nb++;
      buf_sz[bid] = sizes[i];
    }
    assignment[i] = bid;
    for (int32_t a = na; a > 0; --a) { act_id[a] = act_id[a - 1]; act_end[a] = act_end[a - 1]; act_dt[a] = act_dt[a - 1]; }
    act_id[0] = bid; act_end[0] = last[i]; act_dt[0] = dt; ++na;
  }
  *n_buffers = nb;
  free(last); free(act_id); free(act_end); free(act_dt); free(fr_id); free(fr_dt); free(fr_sz); free(buf_sz);
  return 0;
}
