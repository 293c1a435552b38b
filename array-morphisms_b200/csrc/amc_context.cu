// Memory-reuse context: realize/ctx as a device arena (context.scm).
//
// Trace mode: every buffer a plan allocates is allocated normally and
// recorded (dtype, element count, the recorded buffers its producing launch
// reads), in allocation order — the reference's allocation-rec list
// (context.scm:54-78, record! slot of the dispatch vector :95-119).
// finalize: lifetimes are extended to the last reader (compute-last-uses!,
// :282-295), pinned outputs live to the end, and the records are coloured
// greedily by birth order, one pool per dtype, first fit on the free list
// (allocate-buffers, :325-412).  The coloured buffers are laid out in ONE
// device allocation (the arena).
// Replay mode: plans created against the context receive arena sub-buffers
// by allocation counter (get-workspace-buffer, :256-276) — no allocation.
#include <algorithm>
#include <cstring>

#include "amc_internal.h"
#include "amc_plan.h"

namespace amc {

struct AllocRec {
  int32_t dtype;
  int64_t size;
  std::vector<int32_t> inputs;
  bool pinned = false;
};

struct Ctx {
  int mode = 0;  // 0 trace, 1 replay
  std::vector<AllocRec> recs;
  std::unordered_map<uint64_t, int32_t> id_of;  // buffer handle -> allocation id
  int32_t counter = 0;
  std::vector<int32_t> assignment;
  std::vector<int64_t> buf_offset;  // bytes
  std::vector<int64_t> buf_elems;
  std::vector<int32_t> buf_dtype;
  std::shared_ptr<void> arena;
  int64_t arena_bytes = 0;
  int device = 0;
};

static std::mutex g_ctx_mu;
static std::unordered_map<uint64_t, Ctx*> g_ctxs;
static uint64_t g_next_ctx = 1;

static Ctx* ctx_get(uint64_t h) {
  std::lock_guard<std::mutex> l(g_ctx_mu);
  auto it = g_ctxs.find(h);
  return it == g_ctxs.end() ? nullptr : it->second;
}

// Greedy interval colouring by birth order (allocate-buffers).  Per dtype an
// active list (newest first) and a free list; buffers whose lifetime ended
// before record i move to the front of the free list in active-list order,
// and the first free buffer large enough is reused.
static void colour(const std::vector<AllocRec>& recs, std::vector<int32_t>& assignment, std::vector<int64_t>& sizes,
                   std::vector<int32_t>& dtypes) {
  const int32_t n = (int32_t)recs.size();
  std::vector<int32_t> last(n);
  for (int32_t i = 0; i < n; ++i) last[i] = i;
  for (int32_t i = 0; i < n; ++i)
    for (int32_t p : recs[i].inputs)
      if (p >= 0 && p < n && i > last[p]) last[p] = i;
  for (int32_t i = 0; i < n; ++i)
    if (recs[i].pinned) last[i] = n - 1;
  struct Live { int32_t id; int32_t end; };
  struct Free { int32_t id; int64_t size; };
  std::unordered_map<int32_t, std::vector<Live>> active;  // front = newest
  std::unordered_map<int32_t, std::vector<Free>> freel;   // front = first candidate
  assignment.assign(n, -1);
  sizes.clear();
  dtypes.clear();
  for (int32_t i = 0; i < n; ++i) {
    const int32_t dt = recs[i].dtype;
    auto& act = active[dt];
    auto& fr = freel[dt];
    std::vector<Live> keep;
    for (const Live& e : act) {
      if (e.end < i) fr.insert(fr.begin(), Free{e.id, sizes[e.id]});
      else keep.push_back(e);
    }
    act.swap(keep);
    int32_t bid = -1;
    for (size_t k = 0; k < fr.size(); ++k)
      if (fr[k].size >= recs[i].size) {
        bid = fr[k].id;
        fr.erase(fr.begin() + (long)k);
        break;
      }
    if (bid < 0) {
      bid = (int32_t)sizes.size();
      sizes.push_back(recs[i].size);
      dtypes.push_back(dt);
    } else if (recs[i].size > sizes[bid]) {
      sizes[bid] = recs[i].size;
    }
    assignment[i] = bid;
    act.insert(act.begin(), Live{bid, last[i]});
  }
}

int ctx_alloc(void* cp, int32_t dtype, int64_t n, const std::vector<uint64_t>& reads, uint64_t* h) {
  Ctx* c = (Ctx*)cp;
  if (c->mode == 0) {
    int rc = buf_alloc(dtype, n, h);
    if (rc) return rc;
    AllocRec r;
    r.dtype = dtype;
    r.size = n;
    for (uint64_t b : reads) {
      auto it = c->id_of.find(b);
      if (it != c->id_of.end()) r.inputs.push_back(it->second);
    }
    c->id_of[*h] = (int32_t)c->recs.size();
    c->recs.push_back(r);
    return AMC_OK;
  }
  int32_t id = c->counter++;
  if (id >= (int32_t)c->assignment.size())
    return fail(AMC_ERR_STATE, "context replay: allocation id " + std::to_string(id) + " beyond the traced program (" +
                                   std::to_string(c->assignment.size()) + " allocations)");
  int32_t bid = c->assignment[id];
  if (c->buf_dtype[bid] != dtype) return fail(AMC_ERR_STATE, "context replay: dtype mismatch for allocation " + std::to_string(id));
  if (c->buf_elems[bid] < n) return fail(AMC_ERR_STATE, "context replay: buffer too small for allocation " + std::to_string(id));
  Buffer* b = new Buffer();
  b->ptr = (char*)c->arena.get() + c->buf_offset[bid];
  b->dtype = dtype;
  b->nelem = n;
  b->owned = false;
  b->device = c->device;
  b->keepalive = c->arena;
  *h = buf_register(b);
  c->id_of[*h] = id;
  return AMC_OK;
}

int ctx_mode(void* cp) { return ((Ctx*)cp)->mode; }
int32_t ctx_counter(void* cp) { return ((Ctx*)cp)->counter; }

}  // namespace amc

using namespace amc;

extern "C" {

int amc_ctx_create(uint64_t* out) {
  if (!out) return fail(AMC_ERR_INVALID, "amc_ctx_create: null out");
  Ctx* c = new Ctx();
  cudaGetDevice(&c->device);
  std::lock_guard<std::mutex> l(g_ctx_mu);
  *out = g_next_ctx++;
  g_ctxs[*out] = c;
  return AMC_OK;
}

int amc_plan_create_ctx(uint64_t ch, const amc_node* nodes, int32_t n, uint64_t* plan) {
  Ctx* c = ctx_get(ch);
  if (!c) return fail(AMC_ERR_INVALID, "amc_plan_create_ctx: unknown context");
  return plan_create(c, nodes, n, plan);
}

int amc_ctx_pin_output(uint64_t ch, uint64_t ph) {
  Ctx* c = ctx_get(ch);
  Plan* p = plan_get(ph);
  if (!c || !p) return fail(AMC_ERR_INVALID, "amc_ctx_pin_output: unknown context or plan");
  if (c->mode != 0) return fail(AMC_ERR_STATE, "amc_ctx_pin_output: context is not in trace mode");
  for (const amc_view& r : p->results) {
    auto it = c->id_of.find(r.buf);
    if (it != c->id_of.end()) c->recs[it->second].pinned = true;   // a zero-copy result records nothing
  }
  return AMC_OK;
}

// The replay-plan executor (execute-replay-plan, ssa.scm:1519-1654): a plan
// created in replay mode runs again with the arena buffers it was bound to,
// without re-planning.  It must stand where it was created in the replay
// sequence (the counter at its first allocation id); the counter then moves
// past its allocations, as re-creating it would.
int amc_ctx_replay(uint64_t ch, uint64_t ph, void* stream) {
  Ctx* c = ctx_get(ch);
  Plan* p = plan_get(ph);
  if (!c || !p) return fail(AMC_ERR_INVALID, "amc_ctx_replay: unknown context or plan");
  if (p->ctx != (void*)c || !p->ctx_replay) return fail(AMC_ERR_STATE, "amc_ctx_replay: the plan was not created in this context's replay mode");
  if (c->mode != 1) return fail(AMC_ERR_STATE, "amc_ctx_replay: context is not in replay mode");
  if (c->counter != p->ctx_first_id)
    return fail(AMC_ERR_STATE, "amc_ctx_replay: the plan's allocations start at " + std::to_string(p->ctx_first_id) +
                                   " but the context counter is at " + std::to_string(c->counter) + " (reset-context! first)");
  int rc = plan_execute(p, pick_stream(stream));
  if (rc) return rc;
  c->counter += p->ctx_ids;
  return AMC_OK;
}

int amc_ctx_finalize(uint64_t ch) {
  Ctx* c = ctx_get(ch);
  if (!c) return fail(AMC_ERR_INVALID, "amc_ctx_finalize: unknown context");
  if (c->mode != 0) return fail(AMC_ERR_STATE, "finalize-context!: context is not in trace mode");
  if (fault_injected("alloc")) return fail(AMC_ERR_INJECTED, "finalize: injected allocation failure (AMC_FAULT=alloc)");
  colour(c->recs, c->assignment, c->buf_elems, c->buf_dtype);
  int64_t off = 0;
  c->buf_offset.resize(c->buf_elems.size());
  for (size_t b = 0; b < c->buf_elems.size(); ++b) {
    c->buf_offset[b] = off;
    int64_t bytes = c->buf_elems[b] * (int64_t)dtype_size(c->buf_dtype[b]);
    off += (bytes + 255) / 256 * 256;
  }
  c->arena_bytes = off;
  void* p = nullptr;
  if (off > 0) {
    int cur = 0;
    cudaGetDevice(&cur);
    if (cur != c->device) cudaSetDevice(c->device);
    cudaError_t e = cudaMalloc(&p, (size_t)off);
    if (cur != c->device) cudaSetDevice(cur);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc(arena)");
  }
  int dev = c->device;
  c->arena = std::shared_ptr<void>(p, [dev](void* q) {
    if (!q) return;
    int cur = 0;
    cudaGetDevice(&cur);
    if (cur != dev) cudaSetDevice(dev);
    cudaFree(q);
    if (cur != dev) cudaSetDevice(cur);
  });
  c->mode = 1;
  c->counter = 0;
  c->id_of.clear();
  return AMC_OK;
}

int amc_ctx_reset(uint64_t ch) {
  Ctx* c = ctx_get(ch);
  if (!c) return fail(AMC_ERR_INVALID, "amc_ctx_reset: unknown context");
  if (c->mode != 1) return fail(AMC_ERR_STATE, "reset-context!: context is not in replay mode");
  c->counter = 0;
  c->id_of.clear();
  return AMC_OK;
}

int amc_ctx_stats(uint64_t ch, int32_t* allocations, int32_t* buffers, int64_t* arena_bytes, int32_t* mode) {
  Ctx* c = ctx_get(ch);
  if (!c) return fail(AMC_ERR_INVALID, "amc_ctx_stats: unknown context");
  if (allocations) *allocations = (int32_t)c->recs.size();
  if (buffers) *buffers = c->mode == 1 ? (int32_t)c->buf_elems.size() : (int32_t)c->recs.size();
  if (arena_bytes) *arena_bytes = c->arena_bytes;
  if (mode) *mode = c->mode;
  return AMC_OK;
}

int amc_ctx_destroy(uint64_t ch) {
  Ctx* c = nullptr;
  {
    std::lock_guard<std::mutex> l(g_ctx_mu);
    auto it = g_ctxs.find(ch);
    if (it == g_ctxs.end()) return fail(AMC_ERR_INVALID, "amc_ctx_destroy: unknown context");
    c = it->second;
    g_ctxs.erase(it);
  }
  delete c;  // the arena is freed when the last sub-buffer referencing it goes
  return AMC_OK;
}

int amc_colour(int32_t n, const int32_t* dtypes, const int64_t* sizes, const int32_t* in_off, const int32_t* inputs,
               const int32_t* pinned, int32_t* assignment, int32_t* n_buffers) {
  if (n < 0 || (n > 0 && (!dtypes || !sizes || !in_off || !assignment)) || !n_buffers)
    return fail(AMC_ERR_INVALID, "amc_colour: bad arguments");
  std::vector<AllocRec> recs(n);
  for (int32_t i = 0; i < n; ++i) {
    recs[i].dtype = dtypes[i];
    recs[i].size = sizes[i];
    for (int32_t k = in_off[i]; k < in_off[i + 1]; ++k) recs[i].inputs.push_back(inputs[k]);
    recs[i].pinned = pinned && pinned[i];
  }
  std::vector<int32_t> asg;
  std::vector<int64_t> sz;
  std::vector<int32_t> dt;
  colour(recs, asg, sz, dt);
  for (int32_t i = 0; i < n; ++i) assignment[i] = asg[i];
  *n_buffers = (int32_t)sz.size();
  return AMC_OK;
}

}  // extern "C"
