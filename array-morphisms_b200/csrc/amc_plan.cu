// The realize planner.  Input: the morphism tree the reference's realize
// would walk (realization.scm:92-115), serialized as amc_node records.
// Output: a list of device launches over buffers fixed at plan creation.
//
// Lowering rules (each keeps the reference's values):
//   - reshape / transpose / slice of a concrete view are zero-copy views
//     (create-view, realization.scm:649-717).  A reshape the strides cannot
//     express (the reference's execute-affine-morphism copy, :849-862) is a
//     copy in logical row-major order.
//   - element-wise nodes stay lazy: a node is a postfix program over strided
//     leaf views broadcast to its shape.  Operands that are themselves lazy
//     are inlined, followed by a store conversion to the operand's dtype, so
//     the fused kernel rounds exactly where the reference materialises.
//     Transposes and slices of lazy nodes move onto their leaves.
//   - a reduction evaluates its (lazy) operand at source coordinates and folds
//     in the reference's order (realization.scm:1309-1388).
//   - im2col without padding is a strided view when the strides allow it;
//     otherwise it, pad, col2im, stack and concat are gather kernels.
//   - matmul / matvec / dot run the double-accumulating GEMM.
//   - the conv pattern reshape(matmul(W, im2col(X))) on one f32 image
//     (detect-conv2d-pattern, realization.scm:136-164) runs the convolution
//     entry, with no column matrix: the implicit-GEMM tensor-core kernel where
//     its shape conditions hold (TF32 operands, 2e-3 of the output scale),
//     else the direct kernel with double accumulation.
//   - attention of contiguous f32 operands with head dim 64 and n a multiple
//     of 128 runs the tensor-core kernel (TF32, 2e-3); every other attention
//     runs the streaming kernel that keeps the reference's rounding.
//   - the polyphase filter bank (a tap reduction of a product of a windowed
//     view and a broadcast filter) runs the streaming FIR kernel.
#include <algorithm>
#include <cstring>
#include <functional>
#include <optional>

#include "amc_internal.h"
#include "amc_plan.h"

namespace amc {

// ------------------------------------------------------------------ views
struct View {
  uint64_t buf = 0;
  int32_t dtype = AMC_F64;
  int32_t rank = 0;
  int64_t shape[AMC_MAX_RANK] = {0};
  int64_t strides[AMC_MAX_RANK] = {0};
  int64_t offset = 0;
};

static int64_t numel(int32_t rank, const int64_t* shape) {
  int64_t n = 1;
  for (int i = 0; i < rank; ++i) n *= shape[i];
  return n;
}

static void row_major(int32_t rank, const int64_t* shape, int64_t* strides) {
  int64_t s = 1;
  for (int i = rank - 1; i >= 0; --i) {
    strides[i] = s;
    s *= shape[i];
  }
}

static bool is_row_major(const View& v) {
  int64_t st[AMC_MAX_RANK];
  row_major(v.rank, v.shape, st);
  for (int i = 0; i < v.rank; ++i)
    if (v.shape[i] != 1 && v.strides[i] != st[i]) return false;
  return true;
}

static bool same_view(const View& a, const View& b) {
  if (a.buf != b.buf || a.dtype != b.dtype || a.rank != b.rank || a.offset != b.offset) return false;
  for (int i = 0; i < a.rank; ++i)
    if (a.shape[i] != b.shape[i] || a.strides[i] != b.strides[i]) return false;
  return true;
}

// Stride-only reshape (merge/split of dims that are laid out compatibly).
static bool try_reshape(const View& v, int32_t nrank, const int64_t* nshape, View& out) {
  out = v;
  out.rank = nrank;
  for (int i = 0; i < nrank; ++i) out.shape[i] = nshape[i];
  int64_t total = numel(v.rank, v.shape);
  if (total != numel(nrank, nshape)) return false;
  if (total == 0) {
    row_major(nrank, nshape, out.strides);
    return true;
  }
  int64_t od[AMC_MAX_RANK], os[AMC_MAX_RANK];
  int on = 0;
  for (int i = 0; i < v.rank; ++i)
    if (v.shape[i] != 1) { od[on] = v.shape[i]; os[on] = v.strides[i]; ++on; }
  int64_t ns[AMC_MAX_RANK];
  int oi = 0, oj = 1, ni = 0, nj = 1;
  while (ni < nrank && oi < on) {
    if (nshape[ni] == 1) { ns[ni] = 0; ++ni; nj = ni + 1; continue; }
    int64_t np = nshape[ni], op = od[oi];
    while (np != op) {
      if (np < op) { if (nj >= nrank) return false; np *= nshape[nj++]; }
      else { if (oj >= on) return false; op *= od[oj++]; }
    }
    for (int ok = oi; ok < oj - 1; ++ok)
      if (os[ok] != od[ok + 1] * os[ok + 1]) return false;
    ns[nj - 1] = os[oj - 1];
    for (int nk = nj - 1; nk > ni; --nk) ns[nk - 1] = ns[nk] * nshape[nk];
    ni = nj++;
    oi = oj++;
  }
  for (; ni < nrank; ++ni) ns[ni] = 0;  // trailing size-1 dims
  for (int i = 0; i < nrank; ++i) out.strides[i] = ns[i];
  return true;
}

// Broadcast a view to a target shape (numpy rules: trailing alignment, size-1
// dims and missing leading dims get stride 0; basic-ops.scm:84-115).
static bool broadcast_to(const View& v, int32_t rank, const int64_t* shape, View& out) {
  if (v.rank > rank) return false;
  out = v;
  out.rank = rank;
  int lead = rank - v.rank;
  for (int d = 0; d < rank; ++d) {
    out.shape[d] = shape[d];
    if (d < lead) { out.strides[d] = 0; continue; }
    int64_t s = v.shape[d - lead];
    if (s == shape[d]) out.strides[d] = v.strides[d - lead];
    else if (s == 1) out.strides[d] = 0;
    else return false;
  }
  return true;
}

// ------------------------------------------------------------------ values
struct Val {
  bool expr = false;
  View view;                   // concrete value
  int32_t dtype = AMC_F64;     // lazy value
  int32_t rank = 0;
  int64_t shape[AMC_MAX_RANK] = {0};
  std::vector<View> leaves;
  std::vector<amc_insn> prog;
  // The buffer of a GEMM result that this value reads through a chain of
  // single-use map nodes only: materialising the value may fold the chain
  // into that GEMM's store (0: none).
  uint64_t fuse_buf = 0;
};

static amc_insn ins(int op, int a = 0, double imm = 0.0) {
  amc_insn I;
  I.op = op;
  I.a = a;
  I.imm = imm;
  return I;
}

// ------------------------------------------------------------------ plan
int Plan::add_slot(int32_t dtype, int64_t n, const std::vector<uint64_t>& reads, uint64_t* h) {
  int rc;
  if (ctx) rc = ctx_alloc(ctx, dtype, n, reads, h);
  else rc = buf_alloc(dtype, n, h);
  if (rc) return rc;
  slots.push_back(*h);
  bytes += (int64_t)n * (int64_t)dtype_size(dtype);
  return AMC_OK;
}

Plan::~Plan() {
  if (graph_exec) cudaGraphExecDestroy(graph_exec);
  for (uint64_t h : slots) buf_release(h);
  for (uint64_t h : held) buf_release(h);
  for (void* p : dev_small) cudaFree(p);
  for (auto& r : results)
    if (r.buf) buf_release(r.buf);
}

struct Builder {
  const amc_node* nodes;
  int32_t n;
  Plan* plan;
  std::vector<std::optional<Val>> memo;
  std::vector<int> uses;   // operand references to each node (+1 for the root)
  std::vector<char> active; // nodes whose build is in progress
  // While the GEMV pair builds its row program: a slot whose producer reads
  // this buffer would run before the buffer is written (watch_hit).
  uint64_t watch_buf = 0;
  bool watch_hit = false;
  // The forward product X w of the last GEMV pair: slots created after the
  // pair that read it (r0_reads).  When none does and it is no result, the
  // pair need not store it (plan_create clears the store pointer).
  uint64_t r0_watch = 0;
  int r0_reads = 0;
  int pairs_built = 0;
  // The GEMV pair planned last: its launch arguments (shared with its step,
  // which reads them at launch), the buffer of X w and the partial sums.
  struct {
    std::shared_ptr<RowPassArgs> args;
    uint64_t r0 = 0, part = 0;
  } pair;
  // The most recent GEMM step, while its result may still take an epilogue.
  struct {
    size_t step = 0;
    uint64_t cbuf = 0, abuf = 0, bbuf = 0;
    GemmArgs g;
  } tail;

  void count_uses() {
    uses.assign(n, 0);
    for (int i = 0; i < n; ++i) {
      const amc_node& nd = nodes[i];
      if (nd.kind == AMC_N_LEAF) continue;
      const int32_t* in = nd.n_in > AMC_NODE_MAX_IN ? nd.in_ext : nd.in;
      if (!in) continue;
      for (int k = 0; k < nd.n_in; ++k)
        if (in[k] >= 0 && in[k] < n) ++uses[in[k]];
    }
    ++uses[n - 1];
  }

  int err(int code, const std::string& m) { return fail(code, "plan: " + m); }

  void* ptr_of(uint64_t h) {
    Buffer* b = buf_get(h);
    return b ? b->ptr : nullptr;
  }

  DLeaf dleaf(const View& v, int rank_check = -1) {
    DLeaf L;
    memset(&L, 0, sizeof L);
    L.ptr = (const char*)ptr_of(v.buf) + v.offset * (int64_t)dtype_size(v.dtype);
    L.dtype = v.dtype;
    for (int d = 0; d < v.rank; ++d) L.strides[d] = v.strides[d];
    (void)rank_check;
    return L;
  }

  int leaf_view(const amc_node& nd, View& v) {
    const amc_view& lv = nd.leaf;
    Buffer* b = buf_get(lv.buf);
    if (!b) return err(AMC_ERR_INVALID, "leaf refers to an unknown buffer");
    if (lv.dtype != b->dtype) return err(AMC_ERR_INVALID, "leaf dtype does not match its buffer");
    if (lv.rank < 0 || lv.rank > AMC_MAX_RANK) return err(AMC_ERR_INVALID, "leaf rank out of range");
    v.buf = lv.buf;
    v.dtype = lv.dtype;
    v.rank = lv.rank;
    v.offset = lv.offset;
    int64_t lo = lv.offset, hi = lv.offset;
    bool empty = false;
    for (int d = 0; d < lv.rank; ++d) {
      v.shape[d] = lv.shape[d];
      v.strides[d] = lv.strides[d];
      if (lv.shape[d] < 0) return err(AMC_ERR_INVALID, "negative extent");
      if (lv.shape[d] == 0) empty = true;
      else if (lv.strides[d] >= 0) hi += (lv.shape[d] - 1) * lv.strides[d];
      else lo += (lv.shape[d] - 1) * lv.strides[d];
    }
    if (!empty && (lo < 0 || hi >= b->nelem)) return err(AMC_ERR_INVALID, "leaf view reaches outside its buffer");
    return AMC_OK;
  }

  // A contiguous output slot of the given dtype/shape.
  int new_slot(int32_t dtype, int32_t rank, const int64_t* shape, const std::vector<uint64_t>& reads, View& v) {
    if (watch_buf)
      for (uint64_t r : reads)
        if (r == watch_buf) watch_hit = true;
    if (r0_watch)
      for (uint64_t r : reads)
        if (r == r0_watch) {
          ++r0_reads;
          break;
        }
    uint64_t h = 0;
    int rc = plan->add_slot(dtype, numel(rank, shape), reads, &h);
    if (rc) return rc;
    v = View();
    v.buf = h;
    v.dtype = dtype;
    v.rank = rank;
    for (int d = 0; d < rank; ++d) v.shape[d] = shape[d];
    row_major(rank, shape, v.strides);
    v.offset = 0;
    return AMC_OK;
  }

  static std::vector<uint64_t> reads_of(const std::vector<View>& vs) {
    std::vector<uint64_t> r;
    for (auto& v : vs) r.push_back(v.buf);
    return r;
  }

  Val as_expr(const Val& x) {
    if (x.expr) return x;
    Val e;
    e.expr = true;
    e.dtype = x.view.dtype;
    e.rank = x.view.rank;
    for (int d = 0; d < e.rank; ++d) e.shape[d] = x.view.shape[d];
    e.leaves.push_back(x.view);
    e.prog.push_back(ins(AMC_OP_LOAD, 0));
    return e;
  }

  static void fill_prog(DProg& P, const std::vector<amc_insn>& prog_in, const std::vector<View>& leaves) {
    bool allf = true;
    for (auto& I : prog_in) {
      if (I.op == AMC_OP_ICONST) allf = false;
      if (I.op == AMC_OP_CVT && !dtype_float(I.a)) allf = false;
    }
    for (auto& L : leaves)
      if (!dtype_float(L.dtype)) allf = false;
    P.all_float = allf ? 1 : 0;
    // In an all-float program every value is a double, so a store to f64 is
    // the identity and is dropped (config 1's square-then-add carries two).
    std::vector<amc_insn> prog;
    for (auto& I : prog_in)
      if (!(allf && I.op == AMC_OP_CVT && I.a == AMC_F64)) prog.push_back(I);
    P.n = (int32_t)prog.size();
    int sp = 0, mx = 0;
    for (auto& I : prog) {
      if (I.op == AMC_OP_LOAD || I.op == AMC_OP_CONST || I.op == AMC_OP_ICONST) ++sp;
      else if (I.op >= AMC_OP_ADD) --sp;   // binary operators and comparisons pop one
      mx = sp > mx ? sp : mx;
    }
    P.max_depth = mx;
    for (size_t i = 0; i < prog.size(); ++i) P.code[i] = prog[i];
  }

  // Materialise a value into a fresh contiguous slot.
  // Fold an expression over the result of the GEMM step just emitted into
  // that step: allowed when the expression is the GEMM result's only reader
  // (fuse_buf, tracked through single-use nodes), no step came after the
  // GEMM, and the expression reads the result exactly once, as the whole
  // row-major (M, N) array in its own element order.
  int try_fuse_gemm(const Val& e, View& out, bool& done) {
    done = false;
    if (!e.expr || !e.fuse_buf || e.fuse_buf != tail.cbuf || plan->steps.size() != tail.step + 1) return AMC_OK;
    const int64_t total = numel(e.rank, e.shape);
    if (total == 0 || total != tail.g.M * tail.g.N || tail.g.alpha != 1.0 || tail.g.beta != 0.0) return AMC_OK;
    int gl = -1;
    for (size_t l = 0; l < e.leaves.size(); ++l)
      if (e.leaves[l].buf == tail.cbuf) {
        if (gl >= 0) return AMC_OK;
        gl = (int)l;
      }
    if (gl < 0) return AMC_OK;
    const View& L = e.leaves[gl];
    if (L.offset != 0 || L.dtype != tail.g.c_dtype || L.rank != e.rank) return AMC_OK;
    int64_t rm[AMC_MAX_RANK];
    row_major(e.rank, e.shape, rm);
    for (int d = 0; d < e.rank; ++d)
      if (e.shape[d] > 1 && L.strides[d] != rm[d]) return AMC_OK;
    // the epilogue writes while the GEMM reads A and B: keep them live
    std::vector<uint64_t> reads = reads_of(e.leaves);
    reads.push_back(tail.abuf);
    reads.push_back(tail.bbuf);
    int rc = new_slot(e.dtype, e.rank, e.shape, reads, out);
    if (rc) return rc;
    GemmEpiArgs ga;
    memset(&ga, 0, sizeof ga);
    ga.g = tail.g;
    MapArgs& a = ga.map;
    a.rank = e.rank;
    for (int d = 0; d < e.rank; ++d) a.shape[d] = e.shape[d];
    a.total = total;
    a.nleaf = (int32_t)e.leaves.size();
    for (size_t l = 0; l < e.leaves.size(); ++l) a.leaf[l] = dleaf(e.leaves[l]);
    fill_prog(a.prog, e.prog, e.leaves);
    a.out = ptr_of(out.buf);
    a.out_dtype = e.dtype;
    collapse_map(a);
    ga.leaf = gl;
    plan->steps.back() = [ga](cudaStream_t s) { return launch_gemm_epi(ga, s); };
    tail.cbuf = 0;
    done = true;
    return AMC_OK;
  }

  int materialize(const Val& x, View& out, bool may_fuse = false) {
    if (may_fuse) {
      bool done = false;
      int rc = try_fuse_gemm(x, out, done);
      if (rc || done) return rc;
    }
    Val e = as_expr(x);
    int rc = new_slot(e.dtype, e.rank, e.shape, reads_of(e.leaves), out);
    if (rc) return rc;
    MapArgs a;
    memset(&a, 0, sizeof a);
    a.rank = e.rank;
    for (int d = 0; d < e.rank; ++d) a.shape[d] = e.shape[d];
    a.total = numel(e.rank, e.shape);
    a.nleaf = (int32_t)e.leaves.size();
    for (size_t l = 0; l < e.leaves.size(); ++l) a.leaf[l] = dleaf(e.leaves[l]);
    fill_prog(a.prog, e.prog, e.leaves);
    a.out = ptr_of(out.buf);
    a.out_dtype = e.dtype;
    collapse_map(a);
    plan->steps.push_back([a](cudaStream_t s) { return launch_map(a, s); });
    plan->launches += 1;
    return AMC_OK;
  }

  // Merge adjacent dims that every leaf (and the contiguous output) walks
  // linearly; drops size-1 dims.
  static void collapse_map(MapArgs& a) {
    int r = 0;
    int64_t sh[AMC_MAX_RANK];
    int64_t st[kMaxLeaves][AMC_MAX_RANK];
    for (int d = 0; d < a.rank; ++d) {
      if (a.shape[d] == 1) continue;
      if (r > 0) {
        bool ok = true;
        for (int l = 0; l < a.nleaf; ++l)
          if (st[l][r - 1] != a.leaf[l].strides[d] * a.shape[d]) ok = false;
        if (ok) {
          sh[r - 1] *= a.shape[d];
          for (int l = 0; l < a.nleaf; ++l) st[l][r - 1] = a.leaf[l].strides[d];
          continue;
        }
      }
      sh[r] = a.shape[d];
      for (int l = 0; l < a.nleaf; ++l) st[l][r] = a.leaf[l].strides[d];
      ++r;
    }
    if (r == 0) {
      r = 1;
      sh[0] = 1;
      for (int l = 0; l < a.nleaf; ++l) st[l][0] = 0;
    }
    a.rank = r;
    for (int d = 0; d < r; ++d) {
      a.shape[d] = sh[d];
      for (int l = 0; l < a.nleaf; ++l) a.leaf[l].strides[d] = st[l][d];
    }
    for (int d = r; d < AMC_MAX_RANK; ++d) {
      a.shape[d] = 1;
      for (int l = 0; l < a.nleaf; ++l) a.leaf[l].strides[d] = 0;
    }
  }

  int concrete(int idx, View& out) {
    Val v;
    int rc = get(idx, v);
    if (rc) return rc;
    if (!v.expr) { out = v.view; return AMC_OK; }
    rc = materialize(v, out, uses[idx] == 1);
    if (rc) return rc;
    memo[idx] = Val();
    memo[idx]->view = out;
    return AMC_OK;
  }

  // Append the program of operand value x (broadcast to shape) into e.
  bool inline_operand(Val& e, const Val& x, int32_t rank, const int64_t* shape) {
    Val xe = as_expr(x);
    std::vector<int> remap;
    for (auto& L : xe.leaves) {
      View b;
      if (!broadcast_to(L, rank, shape, b)) return false;
      int found = -1;
      for (size_t k = 0; k < e.leaves.size(); ++k)
        if (same_view(e.leaves[k], b)) { found = (int)k; break; }
      if (found < 0) {
        if ((int)e.leaves.size() >= kMaxLeaves) return false;
        e.leaves.push_back(b);
        found = (int)e.leaves.size() - 1;
      }
      remap.push_back(found);
    }
    if (e.prog.size() + xe.prog.size() + 1 > AMC_PROG_MAX) return false;
    for (auto I : xe.prog) {
      if (I.op == AMC_OP_LOAD) I.a = remap[I.a];
      e.prog.push_back(I);
    }
    if (x.expr) e.prog.push_back(ins(AMC_OP_CVT, x.dtype));
    return true;
  }

  // A node program over nd.n_in operands must load only those operands, stay
  // within the stack and leave exactly one value.
  int check_prog(const amc_node& nd) {
    if (!nd.prog || nd.prog_len <= 0 || nd.prog_len > AMC_PROG_MAX) return err(AMC_ERR_INVALID, "node without a program");
    {
      int sp = 0;
      for (int i = 0; i < nd.prog_len; ++i) {
        int op = nd.prog[i].op;
        if (op == AMC_OP_LOAD) { if (nd.prog[i].a < 0 || nd.prog[i].a >= nd.n_in) return err(AMC_ERR_INVALID, "LOAD of a missing operand"); ++sp; }
        else if (op == AMC_OP_CONST || op == AMC_OP_ICONST) ++sp;
        else if (op == AMC_OP_CVT) { if (sp < 1 || !dtype_valid(nd.prog[i].a)) return err(AMC_ERR_INVALID, "bad CVT"); }
        else if (op >= AMC_OP_NEG && op <= AMC_OP_TANH) { if (sp < 1) return err(AMC_ERR_INVALID, "stack underflow"); }
        else if (op >= AMC_OP_ADD && op <= AMC_OP_LE) { if (sp < 2) return err(AMC_ERR_INVALID, "stack underflow"); --sp; }
        else return err(AMC_ERR_INVALID, "unknown opcode");
        if (sp > AMC_STACK_MAX) return err(AMC_ERR_INVALID, "program needs too deep a stack");
      }
      if (sp != 1) return err(AMC_ERR_INVALID, "program must leave one value");
    }
    return AMC_OK;
  }

  int node_map(const amc_node& nd, Val& out) {
    if (nd.n_in < 1 || nd.n_in > AMC_NODE_MAX_IN) return err(AMC_ERR_INVALID, "map node needs 1..4 operands");
    int prc = check_prog(nd);
    if (prc) return prc;
    Val e;
    e.expr = true;
    e.dtype = nd.dtype;
    e.rank = nd.rank;
    for (int d = 0; d < nd.rank; ++d) e.shape[d] = nd.shape[d];
    // operand programs become sub-programs; record where each starts
    std::vector<std::vector<amc_insn>> sub(nd.n_in);
    bool plain = false;   // an operand fits neither inlined nor as one more leaf
    for (int k = 0; k < nd.n_in && !plain; ++k) {
      Val x;
      int rc = get(nd.in[k], x);
      if (rc) return rc;
      Val trial = e;
      trial.prog.clear();
      if (!inline_operand(trial, x, e.rank, e.shape)) {
        View m;
        if (x.expr) {
          rc = materialize(x, m, uses[nd.in[k]] == 1);
          if (rc) return rc;
        } else {
          m = x.view;
        }
        Val mv;
        mv.view = m;
        trial = e;
        trial.prog.clear();
        // still no room when the operands before it took every leaf slot
        // (a long chain such as a fold over a batch): fall back below
        if (!inline_operand(trial, mv, e.rank, e.shape)) {
          plain = true;
          break;
        }
      }
      e.leaves = trial.leaves;
      sub[k] = trial.prog;
      if (!e.fuse_buf && x.fuse_buf && uses[nd.in[k]] == 1) e.fuse_buf = x.fuse_buf;
    }
    // splice: each LOAD k of the node program becomes operand k's sub-program
    std::vector<amc_insn> prog;
    if (!plain)
      for (int i = 0; i < nd.prog_len; ++i) {
        const amc_insn& I = nd.prog[i];
        if (I.op == AMC_OP_LOAD) prog.insert(prog.end(), sub[I.a].begin(), sub[I.a].end());
        else prog.push_back(I);
      }
    if (plain || prog.size() > AMC_PROG_MAX) {
      // too long, or too many leaves: materialise the operands and use plain loads
      e.leaves.clear();
      e.fuse_buf = 0;
      std::vector<View> ms;
      for (int k = 0; k < nd.n_in; ++k) {
        View m;
        int rc = concrete(nd.in[k], m);
        if (rc) return rc;
        View b;
        if (!broadcast_to(m, e.rank, e.shape, b)) return err(AMC_ERR_INVALID, "operand shape does not broadcast");
        e.leaves.push_back(b);
      }
      prog.assign(nd.prog, nd.prog + nd.prog_len);
    }
    e.prog = prog;
    out = e;
    return AMC_OK;
  }

  int node_view(const amc_node& nd, Val& out) {
    if (nd.n_in != 1) return err(AMC_ERR_INVALID, "view node needs one operand");
    Val x;
    int rc = get(nd.in[0], x);
    if (rc) return rc;
    int32_t r = x.expr ? x.rank : x.view.rank;
    const int64_t* xs = x.expr ? x.shape : x.view.shape;
    auto apply = [&](View& v) -> bool {
      if (nd.kind == AMC_N_TRANSPOSE) {
        View t = v;
        for (int d = 0; d < r; ++d) {
          int p = (int)nd.iparam[d];
          t.shape[d] = v.shape[p];
          t.strides[d] = v.strides[p];
        }
        v = t;
        return true;
      }
      // slice: strides scale by step, offset moves by start
      for (int d = 0; d < r; ++d) {
        v.offset += nd.iparam[d] * v.strides[d];
        v.strides[d] *= nd.iparam[8 + d];
        v.shape[d] = nd.shape[d];
      }
      return true;
    };
    if (nd.kind == AMC_N_TRANSPOSE) {
      if (nd.rank != r) return err(AMC_ERR_INVALID, "transpose rank mismatch");
      std::vector<int> seen(r, 0);
      for (int d = 0; d < r; ++d) {
        int p = (int)nd.iparam[d];
        if (p < 0 || p >= r || seen[p]) return err(AMC_ERR_INVALID, "invalid permutation");
        seen[p] = 1;
      }
    } else {
      if (nd.rank != r) return err(AMC_ERR_INVALID, "slice rank mismatch");
      for (int d = 0; d < r; ++d) {
        int64_t st = nd.iparam[d], step = nd.iparam[8 + d];
        if (step <= 0 || st < 0 || (xs[d] > 0 && st >= xs[d]) || nd.shape[d] < 0 ||
            (nd.shape[d] > 0 && st + (nd.shape[d] - 1) * step >= xs[d]))
          return err(AMC_ERR_INVALID, "slice out of range");
      }
    }
    if (!x.expr) {
      out = x;
      apply(out.view);
      return AMC_OK;
    }
    out = x;
    for (auto& L : out.leaves) apply(L);
    for (int d = 0; d < nd.rank; ++d) out.shape[d] = nd.shape[d];
    return AMC_OK;
  }

  // reshape(matmul(W, im2col(X))) with X one (C, H, W) f32 image: the
  // convolution entry computes it without the column matrix.  `done` stays
  // false (and nothing is planned) for any other tree.
  int try_conv(const amc_node& nd, Val& out, bool& done) {
    done = false;
    const amc_node& mm = nodes[nd.in[0]];
    if (mm.kind != AMC_N_MATMUL || mm.n_in != 2 || mm.in[1] < 0 || mm.in[1] >= nd.in[0]) return AMC_OK;
    const amc_node& ic = nodes[mm.in[1]];
    if (ic.kind != AMC_N_IM2COL || ic.n_in != 1 || nd.dtype != AMC_F32 || mm.dtype != AMC_F32 || ic.dtype != AMC_F32)
      return AMC_OK;
    const int32_t KH = ic.iparam[0], KW = ic.iparam[1], SH = ic.iparam[2], SW = ic.iparam[3], PH = ic.iparam[4],
                  PW = ic.iparam[5];
    if (KH <= 0 || KW <= 0 || SH <= 0 || SW <= 0 || PH < 0 || PW < 0) return AMC_OK;
    View X, Wt;
    int rc = concrete(ic.in[0], X);
    if (!rc) rc = concrete(mm.in[0], Wt);
    if (rc) return rc;
    if (X.rank != 3 || Wt.rank != 2 || X.dtype != AMC_F32 || Wt.dtype != AMC_F32 || !is_row_major(X) ||
        !is_row_major(Wt))
      return AMC_OK;
    const int64_t C = X.shape[0], H = X.shape[1], Wd = X.shape[2], K = Wt.shape[0];
    if (Wt.shape[1] != C * KH * KW || C > INT32_MAX || H > INT32_MAX || Wd > INT32_MAX || K > INT32_MAX) return AMC_OK;
    const int64_t OH = 1 + (H + 2 * PH - KH) / SH, OW = 1 + (Wd + 2 * PW - KW) / SW;
    if (H + 2 * PH < KH || Wd + 2 * PW < KW || nd.rank != 3 || nd.shape[0] != K || nd.shape[1] != OH ||
        nd.shape[2] != OW)
      return AMC_OK;
    View o;
    rc = new_slot(AMC_F32, 3, nd.shape, {X.buf, Wt.buf}, o);
    if (rc) return rc;
    const float* xp = reinterpret_cast<const float*>((const char*)ptr_of(X.buf) + X.offset * 4);
    const float* wp = reinterpret_cast<const float*>((const char*)ptr_of(Wt.buf) + Wt.offset * 4);
    float* yp = reinterpret_cast<float*>(ptr_of(o.buf));
    const int32_t c = (int32_t)C, h = (int32_t)H, w = (int32_t)Wd, k = (int32_t)K;
    plan->steps.push_back([=](cudaStream_t s) {
      return amc_conv2d_fwd_f32(xp, wp, yp, 1, c, h, w, k, KH, KW, SH, SW, PH, PW, s);
    });
    plan->launches += 3;   // tensor-core path: weights, padded input, kernel
    out = Val();
    out.view = o;
    done = true;
    return AMC_OK;
  }

  int node_reshape(const amc_node& nd, Val& out) {
    if (nd.n_in != 1) return err(AMC_ERR_INVALID, "reshape needs one operand");
    bool conv = false;
    int rc0 = try_conv(nd, out, conv);
    if (rc0 || conv) return rc0;
    Val x;
    int rc = get(nd.in[0], x);
    if (rc) return rc;
    int64_t have = x.expr ? numel(x.rank, x.shape) : numel(x.view.rank, x.view.shape);
    if (have != numel(nd.rank, nd.shape)) return err(AMC_ERR_INVALID, "reshape size mismatch");
    View src;
    if (x.expr) {
      rc = materialize(x, src);
      if (rc) return rc;
    } else {
      src = x.view;
    }
    View v;
    if (!try_reshape(src, nd.rank, nd.shape, v)) {
      // copy in the source's logical order, then view
      Val sv;
      sv.view = src;
      View m;
      rc = materialize(sv, m);
      if (rc) return rc;
      if (!try_reshape(m, nd.rank, nd.shape, v)) return err(AMC_ERR_INVALID, "reshape failed");
    }
    out = Val();
    out.view = v;
    return AMC_OK;
  }

  // ----------------------------------------------------------- reduce
  int node_reduce(const amc_node& nd, Val& out) {
    if (nd.n_in != 1) return err(AMC_ERR_INVALID, "reduce needs one operand");
    Val x;
    int rc = get(nd.in[0], x);
    if (rc) return rc;
    Val e = as_expr(x);
    int op = (int)nd.iparam[0];
    int64_t mask = nd.iparam[1];
    if (op < AMC_RED_SUM || op > AMC_RED_MIN) return err(AMC_ERR_INVALID, "unknown reduction");
    if (!dtype_float(nd.dtype) && (op == AMC_RED_MAX || op == AMC_RED_MIN))
      return err(AMC_ERR_UNSUPPORTED, "integer max/min reduction: the reference stores +-inf into an integer vector and fails");
    // the value the reduction reads is the operand node's stored value
    if (x.expr) {
      if (e.prog.size() + 1 > AMC_PROG_MAX) {
        View m;
        rc = materialize(x, m);
        if (rc) return rc;
        Val mv;
        mv.view = m;
        e = as_expr(mv);
      } else {
        e.prog.push_back(ins(AMC_OP_CVT, x.dtype));
      }
    }
    ReduceArgs a;
    memset(&a, 0, sizeof a);
    a.op = op;
    a.out_dtype = nd.dtype;
    a.src_dtype = e.dtype;
    a.nleaf = (int32_t)e.leaves.size();
    int ko = 0, kr = 0;
    int n_red_big = 0;
    for (int d = 0; d < e.rank; ++d)
      if ((mask & (1LL << d)) && e.shape[d] != 1) ++n_red_big;
    for (int d = 0; d < e.rank; ++d) {
      if (mask & (1LL << d)) {
        // a reduced axis of extent 1 adds nothing to the index (kept when
        // every reduced axis has extent 1, so one remains)
        if (e.shape[d] == 1 && n_red_big > 0) continue;
        if (e.shape[d] == 1 && n_red_big == 0 && kr > 0) continue;
        a.rshape[kr] = e.shape[d];
        for (int l = 0; l < a.nleaf; ++l) a.leaf_r[l][kr] = e.leaves[l].strides[d];
        ++kr;
      } else {
        a.oshape[ko] = e.shape[d];
        ++ko;
      }
    }
    for (int l = 0; l < a.nleaf; ++l) {
      a.leaf_o[l] = dleaf(e.leaves[l]);
      int k = 0;
      for (int d = 0; d < e.rank; ++d)
        if (!(mask & (1LL << d))) a.leaf_o[l].strides[k++] = e.leaves[l].strides[d];
      for (; k < AMC_MAX_RANK; ++k) a.leaf_o[l].strides[k] = 0;
    }
    a.orank = ko;
    a.rrank = kr;
    a.O = numel(ko, a.oshape);
    a.R = numel(kr, a.rshape);
    fill_prog(a.prog, e.prog, e.leaves);
    View o;
    std::vector<uint64_t> reads = reads_of(e.leaves);
    if (pair.args) reads.push_back(pair.part);   // a folded row sum reads the pair's partials
    rc = new_slot(nd.dtype, nd.rank, nd.shape, reads, o);
    if (rc) return rc;
    a.out = ptr_of(o.buf);
    if (try_fold_row_sum(a, e, o, op)) {
      // the folded sum reads the pair's partials, not X w
      if (r0_watch)
        for (uint64_t rb : reads)
          if (rb == r0_watch) {
            --r0_reads;
            break;
          }
      out = Val();
      out.view = o;
      return AMC_OK;
    }
    if (try_fir(a, e)) {
      out = Val();
      out.view = o;
      return AMC_OK;
    }
    size_t need = 0;
    launch_reduce(a, nullptr, nullptr, 0, &need);
    void* scratch = nullptr;
    if (need) {
      View sv;
      int64_t sh[1] = {(int64_t)((need + 7) / 8)};
      rc = new_slot(AMC_F64, 1, sh, {}, sv);
      if (rc) return rc;
      scratch = ptr_of(sv.buf);
    }
    plan->steps.push_back([a, scratch, need](cudaStream_t s) { return launch_reduce(a, s, scratch, need, nullptr); });
    plan->launches += need ? 2 : 1;
    out = Val();
    out.view = o;
    return AMC_OK;
  }

  // Recognise the filter-bank reduction: sum over one axis of
  // fl32(x * h) with x a view whose tap and frame strides coincide.
  bool try_fir(const ReduceArgs& a, const Val& e) {
    if (a.op != AMC_RED_SUM || a.out_dtype != AMC_F32 || a.src_dtype != AMC_F32) return false;
    if (a.nleaf != 2 || a.rrank != 1 || a.orank < 2) return false;
    // program: LOAD, LOAD, MUL, then store conversions to f32 only
    const auto& P = e.prog;
    if (P.size() < 4 || !(P[0].op == AMC_OP_LOAD && P[1].op == AMC_OP_LOAD && P[0].a != P[1].a && P[2].op == AMC_OP_MUL))
      return false;
    for (size_t i = 3; i < P.size(); ++i)
      if (!(P[i].op == AMC_OP_CVT && P[i].a == AMC_F32)) return false;
    if (e.leaves[0].dtype != AMC_F32 || e.leaves[1].dtype != AMC_F32) return false;
    // which leaf is the filter: stride 0 over every kept axis but the last
    int hi = -1;
    for (int l = 0; l < 2; ++l) {
      bool filt = true;
      for (int d = 0; d < a.orank - 1; ++d)
        if (a.leaf_o[l].strides[d] != 0) filt = false;
      if (filt) hi = l;
    }
    if (hi < 0) return false;
    int xi = 1 - hi;
    const int ko = a.orank;
    FirArgs f;
    memset(&f, 0, sizeof f);
    f.taps = (int32_t)a.rshape[0];
    f.branches = (int32_t)a.oshape[ko - 1];
    f.frames = a.oshape[ko - 2];
    if (a.leaf_o[xi].strides[ko - 1] != 1 || a.leaf_o[hi].strides[ko - 1] != 1) return false;
    f.hop = a.leaf_o[xi].strides[ko - 2];
    f.x_tstride = a.leaf_r[xi][0];
    f.h_tstride = a.leaf_r[hi][0];
    // leading kept axes collapse into one batch axis for x (and the output)
    int64_t B = 1, xbs = 0;
    for (int d = ko - 3; d >= 0; --d) {
      int64_t s = a.leaf_o[xi].strides[d];
      if (a.oshape[d] == 1) continue;
      if (B == 1) { xbs = s; B = a.oshape[d]; }
      else if (s == xbs * B) { B *= a.oshape[d]; }
      else return false;
    }
    f.batch = B;
    f.x_bstride = xbs;
    f.x = (const float*)a.leaf_o[xi].ptr;
    f.h = (const float*)a.leaf_o[hi].ptr;
    f.out = (float*)a.out;
    f.o_fstride = f.branches;
    f.o_bstride = f.frames * f.branches;
    if (!fir_supported(f)) return false;
    plan->steps.push_back([f](cudaStream_t s) { return launch_fir(f, s); });
    plan->launches += fir_launches(f);
    plan->used_fir = true;
    return true;
  }

  // ----------------------------------------------------------- structural gathers
  int node_pad(const amc_node& nd, Val& out) {
    View src;
    int rc = concrete(nd.in[0], src);
    if (rc) return rc;
    if (nd.rank != src.rank) return err(AMC_ERR_INVALID, "pad rank mismatch");
    PadArgs a;
    memset(&a, 0, sizeof a);
    a.rank = nd.rank;
    a.mode = (int32_t)nd.iparam[0];
    if (a.mode < AMC_PAD_CONSTANT || a.mode > AMC_PAD_REFLECT) return err(AMC_ERR_INVALID, "unknown pad mode");
    for (int d = 0; d < nd.rank; ++d) {
      a.oshape[d] = nd.shape[d];
      a.sshape[d] = src.shape[d];
      a.sstrides[d] = src.strides[d];
      a.before[d] = nd.iparam[1 + 2 * d];
      if (nd.shape[d] != src.shape[d] + nd.iparam[1 + 2 * d] + nd.iparam[2 + 2 * d]) return err(AMC_ERR_INVALID, "pad shape mismatch");
      if (src.shape[d] == 0 && nd.shape[d] > 0 && a.mode != AMC_PAD_CONSTANT) return err(AMC_ERR_INVALID, "edge/reflect pad of an empty axis");
    }
    a.src = (const char*)ptr_of(src.buf) + src.offset * (int64_t)dtype_size(src.dtype);
    a.src_dtype = src.dtype;
    a.value = nd.fparam[0];
    a.total = numel(nd.rank, nd.shape);
    View o;
    rc = new_slot(nd.dtype, nd.rank, nd.shape, {src.buf}, o);
    if (rc) return rc;
    a.out = ptr_of(o.buf);
    a.out_dtype = nd.dtype;
    plan->steps.push_back([a](cudaStream_t s) { return launch_pad(a, s); });
    plan->launches += 1;
    out = Val();
    out.view = o;
    return AMC_OK;
  }

  int node_im2col(const amc_node& nd, Val& out) {
    View src;
    int rc = concrete(nd.in[0], src);
    if (rc) return rc;
    if (src.rank != 3 && src.rank != 4) return err(AMC_ERR_INVALID, "im2col needs (C,H,W) or (N,C,H,W)");
    bool batched = src.rank == 4;
    int b = batched ? 1 : 0;
    Im2colArgs a;
    memset(&a, 0, sizeof a);
    a.N = batched ? src.shape[0] : 1;
    a.C = src.shape[b];
    a.H = src.shape[b + 1];
    a.W = src.shape[b + 2];
    a.KH = (int32_t)nd.iparam[0]; a.KW = (int32_t)nd.iparam[1];
    a.SH = (int32_t)nd.iparam[2]; a.SW = (int32_t)nd.iparam[3];
    a.PH = (int32_t)nd.iparam[4]; a.PW = (int32_t)nd.iparam[5];
    if (a.KH <= 0 || a.KW <= 0 || a.SH <= 0 || a.SW <= 0 || a.PH < 0 || a.PW < 0) return err(AMC_ERR_INVALID, "bad im2col parameters");
    a.OH = 1 + (a.H + 2 * a.PH - a.KH) / a.SH;
    a.OW = 1 + (a.W + 2 * a.PW - a.KW) / a.SW;
    if (a.OH <= 0 || a.OW <= 0) return err(AMC_ERR_INVALID, "im2col window larger than the padded image");
    // zero-copy when no window touches padding and the strides allow it
    if (a.PH == 0 && a.PW == 0) {
      View v6 = src;
      int k = 0;
      int64_t sN = batched ? src.strides[0] : 0, sC = src.strides[b], sH = src.strides[b + 1], sW = src.strides[b + 2];
      if (batched) { v6.shape[k] = a.N; v6.strides[k++] = sN; }
      v6.shape[k] = a.C; v6.strides[k++] = sC;
      v6.shape[k] = a.KH; v6.strides[k++] = sH;
      v6.shape[k] = a.KW; v6.strides[k++] = sW;
      v6.shape[k] = a.OH; v6.strides[k++] = sH * a.SH;
      v6.shape[k] = a.OW; v6.strides[k++] = sW * a.SW;
      v6.rank = k;
      View v;
      if (try_reshape(v6, nd.rank, nd.shape, v)) {
        out = Val();
        out.view = v;
        return AMC_OK;
      }
    }
    a.sN = batched ? src.strides[0] : 0;
    a.sC = src.strides[b];
    a.sH = src.strides[b + 1];
    a.sW = src.strides[b + 2];
    a.src = (const char*)ptr_of(src.buf) + src.offset * (int64_t)dtype_size(src.dtype);
    a.src_dtype = src.dtype;
    View o;
    rc = new_slot(nd.dtype, nd.rank, nd.shape, {src.buf}, o);
    if (rc) return rc;
    a.out = ptr_of(o.buf);
    a.out_dtype = nd.dtype;
    plan->steps.push_back([a](cudaStream_t s) { return launch_im2col(a, s); });
    plan->launches += 1;
    out = Val();
    out.view = o;
    return AMC_OK;
  }

  int node_col2im(const amc_node& nd, Val& out) {
    View col;
    int rc = concrete(nd.in[0], col);
    if (rc) return rc;
    bool batched = nd.rank == 4;
    if (!((col.rank == 2 && nd.rank == 3) || (col.rank == 3 && nd.rank == 4))) return err(AMC_ERR_INVALID, "col2im rank mismatch");
    // the reference reads col linearly from index 0; make it contiguous
    int64_t rm[AMC_MAX_RANK];
    row_major(col.rank, col.shape, rm);
    bool contig = col.offset == 0;
    for (int d = 0; d < col.rank; ++d)
      if (col.shape[d] != 1 && col.strides[d] != rm[d]) contig = false;
    if (!contig) {
      Val cv;
      cv.view = col;
      rc = materialize(cv, col);
      if (rc) return rc;
    }
    Col2imArgs a;
    memset(&a, 0, sizeof a);
    int b = batched ? 1 : 0;
    a.N = batched ? nd.shape[0] : 1;
    a.C = nd.shape[b];
    a.H = nd.shape[b + 1];
    a.W = nd.shape[b + 2];
    a.KH = (int32_t)nd.iparam[0]; a.KW = (int32_t)nd.iparam[1];
    a.SH = (int32_t)nd.iparam[2]; a.SW = (int32_t)nd.iparam[3];
    a.PH = (int32_t)nd.iparam[4]; a.PW = (int32_t)nd.iparam[5];
    if (a.KH <= 0 || a.KW <= 0 || a.SH <= 0 || a.SW <= 0 || a.PH < 0 || a.PW < 0) return err(AMC_ERR_INVALID, "bad col2im parameters");
    a.OH = 1 + (a.H + 2 * a.PH - a.KH) / a.SH;
    a.OW = 1 + (a.W + 2 * a.PW - a.KW) / a.SW;
    if (col.shape[b] != a.C * a.KH * a.KW) return err(AMC_ERR_INVALID, "col2im: col-rows mismatch");
    if (col.shape[b + 1] != a.OH * a.OW) return err(AMC_ERR_INVALID, "col2im: col-cols mismatch");
    if (batched && col.shape[0] != a.N) return err(AMC_ERR_INVALID, "col2im: batch size mismatch");
    a.col = ptr_of(col.buf);
    a.col_dtype = col.dtype;
    View o;
    rc = new_slot(nd.dtype, nd.rank, nd.shape, {col.buf}, o);
    if (rc) return rc;
    a.out = ptr_of(o.buf);
    a.out_dtype = nd.dtype;
    plan->steps.push_back([a](cudaStream_t s) { return launch_col2im(a, s); });
    plan->launches += 1;
    out = Val();
    out.view = o;
    return AMC_OK;
  }

  int node_route(const amc_node& nd, Val& out) {
    const int32_t* ins_ = nd.n_in > AMC_NODE_MAX_IN ? nd.in_ext : nd.in;
    if (nd.n_in < 1 || !ins_) return err(AMC_ERR_INVALID, "stack/concat needs operands");
    bool stack = nd.kind == AMC_N_STACK;
    int axis = (int)nd.iparam[0];
    if (axis < 0 || axis >= nd.rank) return err(AMC_ERR_INVALID, "stack/concat axis out of range");
    std::vector<DLeaf> ls(nd.n_in);
    std::vector<int64_t> ext(nd.n_in);
    std::vector<uint64_t> reads;
    int64_t cat = 0;
    for (int k = 0; k < nd.n_in; ++k) {
      View v;
      int rc = concrete(ins_[k], v);
      if (rc) return rc;
      int want = stack ? nd.rank - 1 : nd.rank;
      if (v.rank != want) return err(AMC_ERR_INVALID, "stack/concat operand rank mismatch");
      for (int d = 0, j = 0; d < nd.rank; ++d) {
        if (stack && d == axis) continue;
        if (!stack && d == axis) { ++j; continue; }
        if (v.shape[j] != nd.shape[d]) return err(AMC_ERR_INVALID, "stack/concat operand shape mismatch");
        ++j;
      }
      ls[k] = dleaf(v);
      ext[k] = stack ? 1 : v.shape[axis];
      cat += ext[k];
      reads.push_back(v.buf);
    }
    if (stack ? nd.shape[axis] != nd.n_in : nd.shape[axis] != cat) return err(AMC_ERR_INVALID, "stack/concat extent mismatch");
    // operand table in device memory (owned by the plan)
    void* dl = nullptr;
    void* de = nullptr;
    AMC_CUDA(cudaMalloc(&dl, ls.size() * sizeof(DLeaf)));
    plan->dev_small.push_back(dl);
    AMC_CUDA(cudaMalloc(&de, ext.size() * sizeof(int64_t)));
    plan->dev_small.push_back(de);
    AMC_CUDA(cudaMemcpy(dl, ls.data(), ls.size() * sizeof(DLeaf), cudaMemcpyHostToDevice));
    AMC_CUDA(cudaMemcpy(de, ext.data(), ext.size() * sizeof(int64_t), cudaMemcpyHostToDevice));
    RouteArgs a;
    memset(&a, 0, sizeof a);
    a.rank = nd.rank;
    a.axis = axis;
    a.is_stack = stack ? 1 : 0;
    a.nsrc = nd.n_in;
    for (int d = 0; d < nd.rank; ++d) a.oshape[d] = nd.shape[d];
    a.srcs = (const DLeaf*)dl;
    a.extents = (const int64_t*)de;
    a.total = numel(nd.rank, nd.shape);
    View o;
    int rc = new_slot(nd.dtype, nd.rank, nd.shape, reads, o);
    if (rc) return rc;
    a.out = ptr_of(o.buf);
    a.out_dtype = nd.dtype;
    plan->steps.push_back([a](cudaStream_t s) { return launch_route(a, s); });
    plan->launches += 1;
    out = Val();
    out.view = o;
    return AMC_OK;
  }

  // ----------------------------------------------------------- BLAS-shaped nodes
  // batch-fold / batch-scan (batch-ops.scm:278-322) of an element-wise step:
  // one thread per element position runs the n steps in order.
  int node_scan(const amc_node& nd, Val& out) {
    if (nd.n_in != 2) return err(AMC_ERR_INVALID, "scan needs init and the batched operand");
    int rc = check_prog(nd);
    if (rc) return rc;
    View I, X;
    rc = concrete(nd.in[0], I);
    if (!rc) rc = concrete(nd.in[1], X);
    if (rc) return rc;
    if (X.rank < 1 || I.rank != X.rank - 1) return err(AMC_ERR_INVALID, "scan: init must have the element shape");
    for (int d = 0; d < I.rank; ++d)
      if (I.shape[d] != X.shape[d + 1]) return err(AMC_ERR_INVALID, "scan: init must have the element shape");
    if (I.dtype != nd.dtype) return err(AMC_ERR_INVALID, "scan: the accumulator keeps the init dtype");
    const bool keep = nd.iparam[0] != 0;
    const int64_t n = X.shape[0];
    if (n < 1) return err(AMC_ERR_INVALID, "scan over an empty batch");
    const View& R = keep ? X : I;
    if (nd.rank != R.rank) return err(AMC_ERR_INVALID, "scan result shape mismatch");
    for (int d = 0; d < nd.rank; ++d)
      if (nd.shape[d] != R.shape[d]) return err(AMC_ERR_INVALID, "scan result shape mismatch");
    View o;
    rc = new_slot(nd.dtype, nd.rank, nd.shape, {I.buf, X.buf}, o);
    if (rc) return rc;
    View xe = X;   // element 0 of x: drop axis 0
    xe.rank = X.rank - 1;
    for (int d = 0; d < xe.rank; ++d) {
      xe.shape[d] = X.shape[d + 1];
      xe.strides[d] = X.strides[d + 1];
    }
    ScanArgs a;
    memset(&a, 0, sizeof a);
    a.rank = I.rank;
    for (int d = 0; d < I.rank; ++d) a.shape[d] = I.shape[d];
    a.P = numel(I.rank, I.shape);
    a.n = n;
    a.xstep = X.strides[0];
    a.keep = keep ? 1 : 0;
    a.leaf[0] = dleaf(I);
    a.leaf[1] = dleaf(xe);
    fill_prog(a.prog, std::vector<amc_insn>(nd.prog, nd.prog + nd.prog_len), {I, xe});
    a.out = ptr_of(o.buf);
    a.out_dtype = nd.dtype;
    a.acc_dtype = I.dtype;
    plan->steps.push_back([a](cudaStream_t s) { return launch_scan(a, s); });
    plan->launches += 1;
    out = Val();
    out.view = o;
    return AMC_OK;
  }

  // ----------------------------------------------------------- the GEMV pair
  // X w over a row-major X (rows x d), and X^T e where e is an element-wise
  // function of X w's rows: the forward and gradient products of a linear
  // model (ssa-vjp's matmul rule, ssa.scm:922-940, on the MSE program).
  // Both run in one read of X (amc_rowpass.cu).

  // The X operand node of a GEMV (rows x d) . (d x 1 | d), else -1.
  int fwd_gemv_x(int i) const {
    const amc_node& nd = nodes[i];
    if ((nd.kind != AMC_N_MATMUL && nd.kind != AMC_N_MATVEC) || nd.n_in != 2) return -1;
    const amc_node& a = nodes[nd.in[0]];
    const amc_node& b = nodes[nd.in[1]];
    if (a.rank != 2) return -1;
    if (nd.kind == AMC_N_MATMUL && !(b.rank == 2 && b.shape[1] == 1)) return -1;
    if (nd.kind == AMC_N_MATVEC && b.rank != 1) return -1;
    return nd.in[0];
  }

  // The X of a transposed GEMV transpose(X) . (rows x 1 | rows), else -1;
  // *bnode receives the vector operand.
  int bwd_gemv_x(int j, int* bnode) const {
    const amc_node& nd = nodes[j];
    if ((nd.kind != AMC_N_MATMUL && nd.kind != AMC_N_MATVEC) || nd.n_in != 2) return -1;
    const amc_node& t = nodes[nd.in[0]];
    const amc_node& b = nodes[nd.in[1]];
    if (t.kind != AMC_N_TRANSPOSE || t.rank != 2 || t.n_in != 1 || t.iparam[0] != 1 || t.iparam[1] != 0) return -1;
    if (nd.kind == AMC_N_MATMUL && !(b.rank == 2 && b.shape[1] == 1)) return -1;
    if (nd.kind == AMC_N_MATVEC && b.rank != 1) return -1;
    *bnode = nd.in[1];
    return t.in[0];
  }

  // 0: v does not depend on node i; 1: it does, through element-wise nodes
  // of `rows` elements only (maps, and reshapes that keep the row order);
  // -1: through anything else.
  int ew_dep(int v, int i, int64_t rows, std::vector<int8_t>& seen) const {
    if (v == i) return 1;
    if (v < i) return 0;   // operands precede their nodes
    if (seen[v] != 2) return seen[v];
    const amc_node& nd = nodes[v];
    int r = 0;
    if (nd.kind != AMC_N_LEAF) {
      const int32_t* in = nd.n_in > AMC_NODE_MAX_IN ? nd.in_ext : nd.in;
      for (int k = 0; k < nd.n_in && r >= 0; ++k) {
        int d = ew_dep(in[k], i, rows, seen);
        if (d < 0) r = -1;
        else if (d > 0) r = 1;
      }
      if (r > 0 && !((nd.kind == AMC_N_MAP || nd.kind == AMC_N_RESHAPE) && numel(nd.rank, nd.shape) == rows)) r = -1;
    }
    seen[v] = (int8_t)r;
    return r;
  }

  // `self` is the node being built (active by definition).
  bool pair_candidate(int i, int j, int bnode, int self) {
    if (memo[i] || memo[j] || (i != self && active[i]) || (j != self && active[j])) return false;
    const amc_node& xa = nodes[nodes[i].in[0]];
    const int64_t rows = xa.shape[0], d = xa.shape[1];
    if (d < 1 || d > kRowPassMaxD || rows * d < kRowPassMinElems) return false;
    if (!dtype_float(nodes[i].dtype) || !dtype_float(nodes[j].dtype)) return false;
    std::vector<int8_t> seen(n, 2);
    return ew_dep(bnode, i, rows, seen) == 1;
  }

  int try_gemv_pair(int idx, Val& out, bool& done) {
    done = false;
    int xi = fwd_gemv_x(idx);
    if (xi >= 0) {
      for (int j = idx + 1; j < n; ++j) {
        int b = -1;
        if (bwd_gemv_x(j, &b) == xi && pair_candidate(idx, j, b, idx)) {
          int rc = build_gemv_pair(idx, j, b);
          if (rc) return rc;
          if (memo[idx]) {
            out = *memo[idx];
            done = true;
          }
          return AMC_OK;
        }
      }
      return AMC_OK;
    }
    int b = -1;
    int xj = bwd_gemv_x(idx, &b);
    if (xj < 0) return AMC_OK;
    for (int i = 0; i < idx; ++i)
      if (fwd_gemv_x(i) == xj && pair_candidate(i, idx, b, idx)) {
        int rc = build_gemv_pair(i, idx, b);
        if (rc) return rc;
        if (memo[idx]) {
          out = *memo[idx];
          done = true;
        }
        return AMC_OK;
      }
    return AMC_OK;
  }

  // Forward product i = X w, gradient product j = X^T e(b).  Sets memo[i];
  // sets memo[j] unless the row program cannot run inside the pass, in which
  // case the forward product alone is placed before its readers and j is
  // built as an ordinary product.
  int build_gemv_pair(int i, int j, int bnode) {
    const amc_node& fi = nodes[i];
    const amc_node& fj = nodes[j];
    View X, w, XT;
    int rc = concrete(fi.in[0], X);
    if (!rc) rc = concrete(fi.in[1], w);
    if (!rc) rc = concrete(fj.in[0], XT);
    if (rc) return rc;
    const int64_t rows = X.shape[0], d = X.shape[1];
    const bool x_ok = X.rank == 2 && dtype_float(X.dtype) && dtype_float(w.dtype) && X.strides[1] == 1 &&
                      X.strides[0] >= d && w.shape[0] == d && XT.buf == X.buf && XT.offset == X.offset &&
                      XT.rank == 2 && XT.strides[0] == X.strides[1] && XT.strides[1] == X.strides[0];
    if (!x_ok) return AMC_OK;   // not a pair after all: both build as ordinary products
    View r0;
    rc = new_slot(fi.dtype, fi.rank, fi.shape, {X.buf, w.buf}, r0);
    if (rc) return rc;
    GemmArgs g;
    memset(&g, 0, sizeof g);
    g.M = rows; g.N = 1; g.K = d; g.alpha = 1.0; g.beta = 0.0;
    g.A = (const char*)ptr_of(X.buf) + X.offset * (int64_t)dtype_size(X.dtype);
    g.a_dtype = X.dtype; g.sa0 = X.strides[0]; g.sa1 = 1;
    g.B = (const char*)ptr_of(w.buf) + w.offset * (int64_t)dtype_size(w.dtype);
    g.b_dtype = w.dtype; g.sb0 = w.strides[0]; g.sb1 = 0;
    g.C = ptr_of(r0.buf); g.c_dtype = fi.dtype;
    memo[i] = Val();
    memo[i]->view = r0;
    // the row program: built with X w standing as r0
    const size_t s0 = plan->steps.size();
    watch_buf = r0.buf;
    watch_hit = false;
    Val ev;
    rc = get(bnode, ev);
    watch_buf = 0;
    if (rc) return rc;
    Val e = as_expr(ev);
    if (ev.expr) e.prog.push_back(ins(AMC_OP_CVT, ev.dtype));   // the GEMM reads b's stored value
    int rleaf = -1;
    bool ok = !watch_hit && numel(e.rank, e.shape) == rows && (e.rank == 1 || (e.rank == 2 && e.shape[1] == 1)) &&
              (int)e.leaves.size() <= kMaxLeaves && e.prog.size() <= (size_t)AMC_PROG_MAX;
    for (size_t l = 0; ok && l < e.leaves.size(); ++l) {
      const View& L = e.leaves[l];
      if (!dtype_float(L.dtype)) ok = false;
      if (L.buf == r0.buf) {
        if (rleaf >= 0 || L.offset != 0 || (rows > 1 && L.strides[0] != 1)) ok = false;
        rleaf = (int)l;
      }
    }
    for (auto& I : e.prog)
      if (I.op == AMC_OP_ICONST || (I.op == AMC_OP_CVT && !dtype_float(I.a))) ok = false;
    if (!ok || rleaf < 0) {
      // the forward product alone, ahead of the steps that read r0
      plan->steps.insert(plan->steps.begin() + (long)s0, [g](cudaStream_t s) { return launch_gemm_scratch(g, nullptr, s); });
      plan->launches += 1;
      tail.cbuf = 0;
      return AMC_OK;
    }
    RowPassArgs a;
    memset(&a, 0, sizeof a);
    a.fwd = 1; a.acc = 1;
    a.rows = rows; a.d = (int32_t)d;
    a.X = g.A; a.x_dtype = X.dtype; a.ldx = X.strides[0];
    a.w = g.B; a.w_dtype = w.dtype; a.sw = w.strides[0];
    a.r = g.C; a.r_dtype = fi.dtype; a.sr = 1;
    a.alpha = 1.0; a.beta = 0.0;
    a.nleaf = (int32_t)e.leaves.size();
    a.e_rleaf = rleaf;
    for (size_t l = 0; l < e.leaves.size(); ++l) {
      a.leaf[l] = dleaf(e.leaves[l]);
      for (int k = 1; k < AMC_MAX_RANK; ++k) a.leaf[l].strides[k] = 0;
      if (rows == 1) a.leaf[l].strides[0] = 0;
    }
    fill_prog(a.prog, e.prog, e.leaves);
    std::vector<uint64_t> reads = reads_of(e.leaves);
    reads.push_back(X.buf);
    reads.push_back(w.buf);
    View part;
    int64_t psz[1] = {(int64_t)((rowpass_scratch_bytes(a) + 7) / 8)};
    rc = new_slot(AMC_F64, 1, psz, reads, part);
    if (rc) return rc;
    reads.push_back(part.buf);
    View dw;
    rc = new_slot(fj.dtype, fj.rank, fj.shape, reads, dw);
    if (rc) return rc;
    a.partials = (double*)ptr_of(part.buf);
    a.out = ptr_of(dw.buf); a.out_dtype = fj.dtype; a.sout = 1;
    rowpass_prepare(a);
    auto ap = std::make_shared<RowPassArgs>(a);
    plan->steps.push_back([ap](cudaStream_t s) { return launch_rowpass(*ap, s); });
    plan->launches += rowpass_launches(a);
    pair.args = ap;
    pair.r0 = r0.buf;
    pair.part = part.buf;
    ++pairs_built;
    r0_watch = r0.buf;
    r0_reads = 0;
    memo[j] = Val();
    memo[j]->view = dw;
    return AMC_OK;
  }

  // A full sum or mean of (X w - y)^2 over the rows of the GEMV pair planned
  // last (the MSE loss): the pair's pass accumulates it as well, and this
  // node only adds the pair's per-CTA partials.  The program must be the
  // square of one residual whose first operand is X w read row by row.
  bool try_fold_row_sum(const ReduceArgs& r, const Val& e, const View& out, int op) {
    if (!pair.args || !pair.args->closed || !rowpass_pair_tma(*pair.args) || (op != AMC_RED_SUM && op != AMC_RED_MEAN))
      return false;
    RowPassArgs& a = *pair.args;
    if (a.rsum || r.O != 1 || r.R != a.rows || r.rrank != 1 || out.dtype != AMC_F64 || r.src_dtype != AMC_F64 ||
        !r.prog.all_float)
      return false;
    // program: MUL(S, S), S = SUB(LOAD rl, v) (CVT f64 already dropped)
    const DProg& P = r.prog;
    if (P.n != 7 || P.code[2].op != AMC_OP_SUB || P.code[5].op != AMC_OP_SUB || P.code[6].op != AMC_OP_MUL) return false;
    for (int k = 0; k < 3; ++k)
      if (P.code[k].op != P.code[3 + k].op || P.code[k].a != P.code[3 + k].a ||
          (P.code[k].op == AMC_OP_CONST && P.code[k].imm != P.code[3 + k].imm))
        return false;
    if (P.code[0].op != AMC_OP_LOAD) return false;
    const int rl = P.code[0].a;
    if (e.leaves[rl].buf != pair.r0 || e.leaves[rl].offset != 0 || (a.rows > 1 && r.leaf_r[rl][0] != 1)) return false;
    int yl = -1;
    double yc = 0.0;
    if (P.code[1].op == AMC_OP_CONST) {
      yc = P.code[1].imm;
    } else if (P.code[1].op == AMC_OP_LOAD && P.code[1].a != rl) {
      // the y leaf joins the pair's row leaves (strides[0]: along the rows)
      DLeaf L = r.leaf_o[P.code[1].a];
      L.strides[0] = r.leaf_r[P.code[1].a][0];
      for (int k = 1; k < AMC_MAX_RANK; ++k) L.strides[k] = 0;
      for (int l = 0; l < a.nleaf; ++l)
        if (a.leaf[l].ptr == L.ptr && a.leaf[l].dtype == L.dtype && a.leaf[l].strides[0] == L.strides[0]) yl = l;
      if (yl < 0) {
        if (a.nleaf >= kMaxLeaves) return false;
        yl = a.nleaf;
        a.leaf[a.nleaf++] = L;
      }
    } else {
      return false;
    }
    a.rsum = 1;
    a.rsum_y_leaf = yl;
    a.rsum_y_const = yc;
    const double* partials = (const double*)ptr_of(pair.part) + (size_t)rowpass_ctas(a) * a.d;
    const int n = rowpass_ctas(a);
    void* o = ptr_of(out.buf);
    const double div = op == AMC_RED_MEAN ? (double)r.R : 0.0;
    plan->steps.push_back([partials, n, o, div](cudaStream_t s) { return launch_rowsum_finish(partials, n, o, AMC_F64, div, s); });
    plan->launches += 1;
    return true;
  }

  int node_gemm(int idx, Val& out) {
    const amc_node& nd = nodes[idx];
    {
      bool done = false;
      int rc = try_gemv_pair(idx, out, done);
      if (rc || done) return rc;
    }
    if (nd.n_in != 2) return err(AMC_ERR_INVALID, "matmul/matvec/dot need two operands");
    View A, B;
    int rc = concrete(nd.in[0], A);
    if (rc) return rc;
    rc = concrete(nd.in[1], B);
    if (rc) return rc;
    if (!dtype_float(A.dtype) || !dtype_float(B.dtype) || !dtype_float(nd.dtype))
      return err(AMC_ERR_UNSUPPORTED, "matmul/matvec/dot are defined for f32/f64 (blas-compat.scm:104-105)");
    GemmArgs g;
    memset(&g, 0, sizeof g);
    g.alpha = 1.0;
    g.beta = 0.0;
    g.a_dtype = A.dtype;
    g.b_dtype = B.dtype;
    g.c_dtype = nd.dtype;
    g.A = (const char*)ptr_of(A.buf) + A.offset * (int64_t)dtype_size(A.dtype);
    g.B = (const char*)ptr_of(B.buf) + B.offset * (int64_t)dtype_size(B.dtype);
    if (nd.kind == AMC_N_MATMUL) {
      if (A.rank != 2 || B.rank != 2 || A.shape[1] != B.shape[0]) return err(AMC_ERR_INVALID, "matmul shape mismatch");
      g.M = A.shape[0]; g.K = A.shape[1]; g.N = B.shape[1];
      g.sa0 = A.strides[0]; g.sa1 = A.strides[1]; g.sb0 = B.strides[0]; g.sb1 = B.strides[1];
    } else if (nd.kind == AMC_N_MATVEC) {
      if (A.rank != 2 || B.rank != 1 || A.shape[1] != B.shape[0]) return err(AMC_ERR_INVALID, "matvec shape mismatch");
      g.M = A.shape[0]; g.K = A.shape[1]; g.N = 1;
      g.sa0 = A.strides[0]; g.sa1 = A.strides[1]; g.sb0 = B.strides[0]; g.sb1 = 0;
    } else {
      if (A.rank != 1 || B.rank != 1 || A.shape[0] != B.shape[0]) return err(AMC_ERR_INVALID, "dot shape mismatch");
      g.M = 1; g.K = A.shape[0]; g.N = 1;
      g.sa0 = 0; g.sa1 = A.strides[0]; g.sb0 = B.strides[0]; g.sb1 = 0;
    }
    View o;
    rc = new_slot(nd.dtype, nd.rank, nd.shape, {A.buf, B.buf}, o);
    if (rc) return rc;
    if (numel(nd.rank, nd.shape) != g.M * g.N) return err(AMC_ERR_INVALID, "matmul result shape mismatch");
    g.C = ptr_of(o.buf);
    const size_t sbytes = gemm_scratch_bytes(g);
    if (sbytes) {
      // a row-pass product (large matrix-vector shapes): no epilogue fusion
      View sv;
      int64_t sh[1] = {(int64_t)((sbytes + 7) / 8)};
      rc = new_slot(AMC_F64, 1, sh, {A.buf, B.buf}, sv);
      if (rc) return rc;
      void* scratch = ptr_of(sv.buf);
      plan->steps.push_back([g, scratch](cudaStream_t s) { return launch_gemm_scratch(g, scratch, s); });
      plan->launches += gemm_launches(g);
      out = Val();
      out.view = o;
      return AMC_OK;
    }
    RowPassArgs rp;
    if (gemm_as_rowpass(g, rp)) {
      plan->steps.push_back([g](cudaStream_t s) { return launch_gemm_scratch(g, nullptr, s); });
      plan->launches += 1;
      out = Val();
      out.view = o;
      return AMC_OK;
    }
    plan->steps.push_back([g](cudaStream_t s) { return launch_gemm(g, s); });
    plan->launches += 1;
    tail.step = plan->steps.size() - 1;
    tail.cbuf = o.buf;
    tail.abuf = A.buf;
    tail.bbuf = B.buf;
    tail.g = g;
    out = Val();
    out.view = o;
    out.fuse_buf = o.buf;
    return AMC_OK;
  }

  int node_attention(const amc_node& nd, Val& out) {
    if (nd.n_in != 3) return err(AMC_ERR_INVALID, "attention needs Q, K, V");
    View Q, K, V;
    int rc = concrete(nd.in[0], Q);
    if (!rc) rc = concrete(nd.in[1], K);
    if (!rc) rc = concrete(nd.in[2], V);
    if (rc) return rc;
    if (Q.rank < 2 || Q.rank > 4 || K.rank != Q.rank || V.rank != Q.rank) return err(AMC_ERR_INVALID, "attention operands must share rank 2..4");
    if (!dtype_float(Q.dtype) || Q.dtype != K.dtype || Q.dtype != V.dtype) return err(AMC_ERR_UNSUPPORTED, "attention needs f32/f64 operands of one dtype");
    int r = Q.rank;
    AttnArgs a;
    memset(&a, 0, sizeof a);
    a.n = (int32_t)Q.shape[r - 2];
    a.dk = (int32_t)Q.shape[r - 1];
    a.dv = (int32_t)V.shape[r - 1];
    if (K.shape[r - 2] != a.n || K.shape[r - 1] != a.dk || V.shape[r - 2] != a.n) return err(AMC_ERR_INVALID, "attention shape mismatch");
    a.blocks = 1;
    for (int d = 0; d < r - 2; ++d) a.blocks *= Q.shape[d];
    a.dtype = Q.dtype;
    a.scale = nd.fparam[0];
    // per-block base = offset + b * stride[rank-3] (execute-fused-attention, :366-373)
    a.Q = (const char*)ptr_of(Q.buf) + Q.offset * (int64_t)dtype_size(Q.dtype);
    a.K = (const char*)ptr_of(K.buf) + K.offset * (int64_t)dtype_size(K.dtype);
    a.V = (const char*)ptr_of(V.buf) + V.offset * (int64_t)dtype_size(V.dtype);
    a.qb = r > 2 ? Q.strides[r - 3] : 0; a.q0 = Q.strides[r - 2]; a.q1 = Q.strides[r - 1];
    a.kb = r > 2 ? K.strides[r - 3] : 0; a.k0 = K.strides[r - 2]; a.k1 = K.strides[r - 1];
    a.vb = r > 2 ? V.strides[r - 3] : 0; a.v0 = V.strides[r - 2]; a.v1 = V.strides[r - 1];
    View o;
    rc = new_slot(nd.dtype, nd.rank, nd.shape, {Q.buf, K.buf, V.buf}, o);
    if (rc) return rc;
    a.O = ptr_of(o.buf);
    if (a.dtype == AMC_F32 && a.dk == 64 && a.dv == 64 && a.n >= 128 && a.n % 128 == 0 && is_row_major(Q) &&
        is_row_major(K) && is_row_major(V)) {
      plan->steps.push_back([a](cudaStream_t s) {
        bool handled = false;
        int rc = attention_fwd_tc((const float*)a.Q, (const float*)a.K, (const float*)a.V, (float*)a.O, nullptr,
                                  a.blocks, a.n, a.dk, a.dv, (float)a.scale, s, &handled);
        if (rc || handled) return rc;
        return launch_attention_generic(a, s);
      });
      plan->launches += 3;   // V^T, K rounding, kernel
    } else {
      plan->steps.push_back([a](cudaStream_t s) { return launch_attention_generic(a, s); });
      plan->launches += 1;
    }
    out = Val();
    out.view = o;
    return AMC_OK;
  }

  // ----------------------------------------------------------- dispatch
  int get(int i, Val& out) {
    if (i < 0 || i >= n) return err(AMC_ERR_INVALID, "operand index out of range");
    if (memo[i]) { out = *memo[i]; return AMC_OK; }
    const amc_node& nd = nodes[i];
    if (!dtype_valid(nd.dtype)) return err(AMC_ERR_INVALID, "invalid dtype");
    if (nd.rank < 0 || nd.rank > AMC_MAX_RANK) return err(AMC_ERR_INVALID, "rank out of range");
    for (int d = 0; d < nd.rank; ++d)
      if (nd.shape[d] < 0) return err(AMC_ERR_INVALID, "negative extent");
    if (nd.kind != AMC_N_LEAF && nd.n_in <= AMC_NODE_MAX_IN)
      for (int k = 0; k < nd.n_in; ++k)
        if (nd.in[k] < 0 || nd.in[k] >= i) return err(AMC_ERR_INVALID, "operands must precede their node");
    if (nd.kind != AMC_N_LEAF && nd.n_in > AMC_NODE_MAX_IN) {
      if (!nd.in_ext) return err(AMC_ERR_INVALID, "missing operand table");
      for (int k = 0; k < nd.n_in; ++k)
        if (nd.in_ext[k] < 0 || nd.in_ext[k] >= i) return err(AMC_ERR_INVALID, "operands must precede their node");
    }
    Val v;
    int rc = AMC_OK;
    active[i] = 1;
    switch (nd.kind) {
      case AMC_N_LEAF: rc = leaf_view(nd, v.view); break;
      case AMC_N_RESHAPE: rc = node_reshape(nd, v); break;
      case AMC_N_TRANSPOSE:
      case AMC_N_SLICE: rc = node_view(nd, v); break;
      case AMC_N_MAP: rc = node_map(nd, v); break;
      case AMC_N_REDUCE: rc = node_reduce(nd, v); break;
      case AMC_N_PAD: rc = node_pad(nd, v); break;
      case AMC_N_IM2COL: rc = node_im2col(nd, v); break;
      case AMC_N_COL2IM: rc = node_col2im(nd, v); break;
      case AMC_N_STACK:
      case AMC_N_CONCAT: rc = node_route(nd, v); break;
      case AMC_N_MATMUL:
      case AMC_N_MATVEC:
      case AMC_N_DOT: rc = node_gemm(i, v); break;
      case AMC_N_ATTENTION: rc = node_attention(nd, v); break;
      case AMC_N_SCAN: rc = node_scan(nd, v); break;
      case AMC_N_OUTPUTS: rc = err(AMC_ERR_INVALID, "an OUTPUTS node must be the last node and no operand"); break;
      default: rc = err(AMC_ERR_INVALID, "unknown node kind"); break;
    }
    active[i] = 0;
    if (rc) return rc;
    if (nd.kind != AMC_N_MAP && nd.kind != AMC_N_MATMUL && nd.kind != AMC_N_MATVEC && nd.kind != AMC_N_DOT)
      v.fuse_buf = 0;
    memo[i] = v;
    out = v;
    return AMC_OK;
  }
};

static std::mutex g_plans_mu;
static std::unordered_map<uint64_t, Plan*> g_plans;
static uint64_t g_next_plan = 1;

Plan* plan_get(uint64_t h) {
  std::lock_guard<std::mutex> l(g_plans_mu);
  auto it = g_plans.find(h);
  return it == g_plans.end() ? nullptr : it->second;
}

int plan_create(void* ctx, const amc_node* nodes, int32_t n, uint64_t* out) {
  if (!nodes || n <= 0 || !out) return fail(AMC_ERR_INVALID, "amc_plan_create: empty tree");
  if (fault_injected("plan")) return fail(AMC_ERR_INJECTED, "plan: injected failure (AMC_FAULT=plan)");
  Plan* p = new Plan();
  p->ctx = ctx;
  if (ctx && ctx_mode(ctx) == 1) {
    p->ctx_replay = true;
    p->ctx_first_id = ctx_counter(ctx);
  }
  Builder b{nodes, n, p, std::vector<std::optional<Val>>(n)};
  b.count_uses();
  b.active.assign(n, 0);
  // roots: the last node, or every operand of a final OUTPUTS node (the
  // outputs of one program realized together, each shared node once)
  std::vector<int> roots;
  int rc = AMC_OK;
  if (nodes[n - 1].kind == AMC_N_OUTPUTS) {
    const amc_node& on = nodes[n - 1];
    const int32_t* in = on.n_in > AMC_NODE_MAX_IN ? on.in_ext : on.in;
    if (on.n_in < 1 || !in) rc = fail(AMC_ERR_INVALID, "plan: OUTPUTS needs at least one operand");
    for (int k = 0; !rc && k < on.n_in; ++k) {
      if (in[k] < 0 || in[k] >= n - 1) rc = fail(AMC_ERR_INVALID, "plan: OUTPUTS operand out of range");
      else roots.push_back(in[k]);
    }
  } else {
    roots.push_back(n - 1);
  }
  for (size_t k = 0; !rc && k < roots.size(); ++k) {
    Val root;
    rc = b.get(roots[k], root);
    if (rc) break;
    View res;
    if (root.expr) {
      rc = b.materialize(root, res, b.uses[roots[k]] == 1);
      if (rc) break;
      b.memo[roots[k]] = Val();
      b.memo[roots[k]]->view = res;   // a root listed twice is one buffer
    } else {
      res = root.view;
    }
    amc_view r;
    memset(&r, 0, sizeof r);
    r.buf = res.buf;
    r.dtype = res.dtype;
    r.rank = res.rank;
    for (int d = 0; d < res.rank; ++d) { r.shape[d] = res.shape[d]; r.strides[d] = res.strides[d]; }
    r.offset = res.offset;
    buf_retain(res.buf);
    p->results.push_back(r);
  }
  if (!rc && b.pairs_built == 1 && b.pair.args && b.r0_reads == 0) {
    // nothing after the pair reads X w and it is no result: skip its store
    bool is_result = false;
    for (auto& r : p->results) is_result = is_result || r.buf == b.r0_watch;
    if (!is_result) b.pair.args->r = nullptr;
  }
  if (!rc) {
    if (p->ctx_replay) p->ctx_ids = ctx_counter(ctx) - p->ctx_first_id;
    p->result = p->results[0];
    p->result_owned = true;
    // hold leaf buffers for the plan's lifetime
    for (int i = 0; i < n; ++i)
      if (nodes[i].kind == AMC_N_LEAF) { buf_retain(nodes[i].leaf.buf); p->held.push_back(nodes[i].leaf.buf); }
  }
  if (rc) {
    delete p;
    return rc;
  }
  std::lock_guard<std::mutex> l(g_plans_mu);
  *out = g_next_plan++;
  g_plans[*out] = p;
  return AMC_OK;
}

int plan_execute(Plan* p, cudaStream_t s) {
  if (p->graph_exec) {
    AMC_CUDA(cudaGraphLaunch(p->graph_exec, s));
    return AMC_OK;
  }
  for (auto& st : p->steps) {
    int rc = st(s);
    if (rc) return rc;
  }
  return AMC_OK;
}

}  // namespace amc

using namespace amc;

extern "C" {

int amc_plan_create(const amc_node* nodes, int32_t n, uint64_t* plan) { return plan_create(nullptr, nodes, n, plan); }

int amc_plan_execute(uint64_t h, void* stream) {
  Plan* p = plan_get(h);
  if (!p) return fail(AMC_ERR_INVALID, "amc_plan_execute: unknown plan");
  return plan_execute(p, pick_stream(stream));
}

int amc_plan_result(uint64_t h, amc_view* out) {
  Plan* p = plan_get(h);
  if (!p || !out) return fail(AMC_ERR_INVALID, "amc_plan_result: unknown plan");
  *out = p->result;
  buf_retain(p->result.buf);  // the caller owns one reference
  return AMC_OK;
}

int amc_plan_result_count(uint64_t h, int32_t* n) {
  Plan* p = plan_get(h);
  if (!p || !n) return fail(AMC_ERR_INVALID, "amc_plan_result_count: unknown plan");
  *n = (int32_t)p->results.size();
  return AMC_OK;
}

int amc_plan_result_at(uint64_t h, int32_t i, amc_view* out) {
  Plan* p = plan_get(h);
  if (!p || !out) return fail(AMC_ERR_INVALID, "amc_plan_result_at: unknown plan");
  if (i < 0 || i >= (int32_t)p->results.size()) return fail(AMC_ERR_INVALID, "amc_plan_result_at: index out of range");
  *out = p->results[i];
  buf_retain(out->buf);  // the caller owns one reference
  return AMC_OK;
}

int amc_plan_stats(uint64_t h, int32_t* launches, int32_t* buffers, int64_t* bytes) {
  Plan* p = plan_get(h);
  if (!p) return fail(AMC_ERR_INVALID, "amc_plan_stats: unknown plan");
  if (launches) *launches = p->launches;
  if (buffers) *buffers = (int32_t)p->slots.size();
  if (bytes) *bytes = p->bytes;
  return AMC_OK;
}

int amc_plan_capture_graph(uint64_t h, void* stream) {
  Plan* p = plan_get(h);
  if (!p) return fail(AMC_ERR_INVALID, "amc_plan_capture_graph: unknown plan");
  if (p->graph_exec) return AMC_OK;
  cudaStream_t s = pick_stream(stream);
  AMC_CUDA(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
  int rc = AMC_OK;
  for (auto& st : p->steps) {
    rc = st(s);
    if (rc) break;
  }
  cudaGraph_t g = nullptr;
  cudaError_t e = cudaStreamEndCapture(s, &g);
  if (rc) { if (g) cudaGraphDestroy(g); return rc; }
  if (e != cudaSuccess) return cuda_fail(e, "cudaStreamEndCapture");
  e = cudaGraphInstantiate(&p->graph_exec, g, 0);
  cudaGraphDestroy(g);
  if (e != cudaSuccess) { p->graph_exec = nullptr; return cuda_fail(e, "cudaGraphInstantiate"); }
  return AMC_OK;
}

int amc_plan_destroy(uint64_t h) {
  Plan* p = nullptr;
  {
    std::lock_guard<std::mutex> l(g_plans_mu);
    auto it = g_plans.find(h);
    if (it == g_plans.end()) return fail(AMC_ERR_INVALID, "amc_plan_destroy: unknown plan");
    p = it->second;
    g_plans.erase(it);
  }
  delete p;
  return AMC_OK;
}

}  // extern "C"
