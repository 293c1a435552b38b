// Fixed-order sum over the GPUs of one node through NVLink peer memory: the
// reduction that crosses the batch axis of a sharded workload (the conv weight
// gradient, the regression gradient; batch-ops.scm:241-254 reduces the
// batch's per-element results in index order).
//
// Every rank owns one allocation, exported by CUDA IPC and opened by every
// other rank of the node:
//   flags[world]                 epoch of the last partial that rank q pushed here
//   slots[2][world][max_elems]   the partials of rank q for even / odd epochs
// A sum at epoch e:
//   push   each rank writes its partial into slot[e % 2][rank] of every rank's
//          allocation (peer stores over NVLink), then fences at system scope;
//   signal one thread stores e into flags[rank] of every rank (release,
//          system scope);
//   wait   each CTA polls its own flags until every rank has signalled e
//          (acquire, system scope; bounded: on expiry it records
//          AMC_ERR_TIMEOUT and returns);
//   sum    out[i] = sum over q = 0 .. world-1, in that order, of slot[e%2][q][i],
//          accumulated in double and stored as the dtype: identical on every
//          rank and every run, whatever the collective's timing.
// Two slots suffice: a rank starts epoch e+2 only after every rank signalled
// e+1, which each does after finishing its sum of epoch e.
// No kernel waits on another kernel of the same GPU; no multicast or
// tensor-memory access is involved, only plain peer loads and stores.
#include <algorithm>
#include <cstring>

#include "amc_internal.h"

namespace amc {

namespace {

__device__ int g_dist_error;
constexpr long long kDistWaitLimit = 1ll << 26;   // polls (with back-off) before a wait gives up

struct PeerGroup {
  int rank = 0, world = 1, device = 0;
  int64_t max_elems = 0;          // per slot, in 8-byte elements
  char* base = nullptr;           // this rank's allocation
  size_t bytes = 0;
  std::vector<char*> peer;        // every rank's allocation (own included), as mapped here
  int64_t epoch = 0;
  bool opened = false;
};

constexpr size_t kFlagBytes = 256;   // flags area (up to 32 ranks), keeps the slots 256-byte aligned
constexpr int kDistThreads = 128;

std::mutex g_groups_mu;
std::unordered_map<uint64_t, PeerGroup*> g_groups;
uint64_t g_next_group = 1;

PeerGroup* group_get(uint64_t h) {
  std::lock_guard<std::mutex> l(g_groups_mu);
  auto it = g_groups.find(h);
  return it == g_groups.end() ? nullptr : it->second;
}

struct PushArgs {
  const void* src;
  int64_t n;            // elements
  int32_t esize;        // 4 or 8
  int32_t world;
  int64_t slot_off;     // byte offset of slot[e % 2][rank] in every allocation
  char* peer[32];
};

__global__ void __launch_bounds__(kDistThreads) k_peer_push(const __grid_constant__ PushArgs a) {
  const long long nb = a.n * a.esize;
  const long long tid = (long long)blockIdx.x * blockDim.x + threadIdx.x, nthr = (long long)gridDim.x * blockDim.x;
  // 16-byte moves where the size allows, then the tail in elements
  const long long n16 = nb / 16;
  const int4* s16 = (const int4*)a.src;
  for (int q = 0; q < a.world; ++q) {
    int4* d16 = (int4*)(a.peer[q] + a.slot_off);
    for (long long i = tid; i < n16; i += nthr) d16[i] = s16[i];
    const char* s = (const char*)a.src;
    char* d = a.peer[q] + a.slot_off;
    for (long long i = n16 * 16 + tid; i < nb; i += nthr) d[i] = s[i];
  }
  __threadfence_system();   // this thread's peer stores before the signal of the next launch
}

struct SumArgs {
  void* out;
  int64_t n;
  int32_t dtype, world, rank;
  int64_t epoch;
  int64_t slot_off0;    // byte offset of slot[e % 2][0] in this rank's allocation
  int64_t slot_stride;  // bytes between ranks' slots
  char* base;           // this rank's allocation
  volatile unsigned long long* flags_local;
  char* peer[32];
};

__device__ __forceinline__ unsigned long long ld_acquire_sys(const volatile unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__global__ void __launch_bounds__(kDistThreads) k_peer_signal_sum(const __grid_constant__ SumArgs a) {
  __shared__ int ok;
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    __threadfence_system();
    for (int q = 0; q < a.world; ++q)
      st_release_sys((unsigned long long*)(a.peer[q]) + a.rank, (unsigned long long)a.epoch);
  }
  if (threadIdx.x == 0) {
    int good = 1;
    for (int q = 0; q < a.world && good; ++q) {
      long long i = 0;
      while (ld_acquire_sys(a.flags_local + q) < (unsigned long long)a.epoch) {
        if (++i > kDistWaitLimit) { good = 0; break; }
        if (i > 64) __nanosleep(64);
      }
    }
    if (!good) atomicExch(&g_dist_error, AMC_ERR_TIMEOUT);
    ok = good;
  }
  __syncthreads();
  if (!ok) return;
  const long long tid = (long long)blockIdx.x * blockDim.x + threadIdx.x, nthr = (long long)gridDim.x * blockDim.x;
  const char* s0 = a.base + a.slot_off0;
  for (long long i = tid; i < a.n; i += nthr) {
    double acc = 0.0;
    for (int q = 0; q < a.world; ++q) {
      const char* sq = s0 + q * a.slot_stride;
      acc += a.dtype == AMC_F32 ? (double)((const volatile float*)sq)[i] : ((const volatile double*)sq)[i];
    }
    if (a.dtype == AMC_F32) ((float*)a.out)[i] = (float)acc;
    else ((double*)a.out)[i] = acc;
  }
}

}  // namespace

int dist_check_error() {
  int e = 0;
  AMC_CUDA(cudaMemcpyFromSymbol(&e, g_dist_error, sizeof(int)));
  if (e) {
    int z = 0;
    AMC_CUDA(cudaMemcpyToSymbol(g_dist_error, &z, sizeof(int)));
    return fail(e, "peer sum: a bounded wait for another rank's partial gave up");
  }
  return AMC_OK;
}

}  // namespace amc

using namespace amc;

extern "C" {

int amc_peer_group_create(int32_t rank, int32_t world, int64_t max_elems, uint64_t* group, void* handle_out) {
  if (!group || !handle_out || world < 1 || world > 32 || rank < 0 || rank >= world || max_elems < 1)
    return fail(AMC_ERR_INVALID, "amc_peer_group_create: rank in [0, world), world 1..32, max_elems >= 1");
  PeerGroup* g = new PeerGroup();
  g->rank = rank;
  g->world = world;
  g->max_elems = (max_elems + 31) / 32 * 32;
  cudaGetDevice(&g->device);
  g->bytes = kFlagBytes + (size_t)2 * world * g->max_elems * 8;
  cudaError_t e = cudaMalloc(&g->base, g->bytes);
  if (e != cudaSuccess) { delete g; return cuda_fail(e, "cudaMalloc(peer group)"); }
  e = cudaMemset(g->base, 0, g->bytes);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();   // zeroed flags before any peer can map them
  if (e == cudaSuccess) e = cudaIpcGetMemHandle((cudaIpcMemHandle_t*)handle_out, g->base);
  if (e != cudaSuccess) { cudaFree(g->base); delete g; return cuda_fail(e, "cudaIpcGetMemHandle(peer group)"); }
  std::lock_guard<std::mutex> l(g_groups_mu);
  *group = g_next_group++;
  g_groups[*group] = g;
  return AMC_OK;
}

int amc_peer_group_open(uint64_t h, const void* handles) {
  PeerGroup* g = group_get(h);
  if (!g || !handles) return fail(AMC_ERR_INVALID, "amc_peer_group_open: unknown group");
  if (g->opened) return fail(AMC_ERR_STATE, "amc_peer_group_open: already open");
  g->peer.assign(g->world, nullptr);
  for (int q = 0; q < g->world; ++q) {
    if (q == g->rank) { g->peer[q] = g->base; continue; }
    cudaIpcMemHandle_t hd;
    memcpy(&hd, (const char*)handles + (size_t)q * sizeof(cudaIpcMemHandle_t), sizeof hd);
    void* p = nullptr;
    cudaError_t e = cudaIpcOpenMemHandle(&p, hd, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return cuda_fail(e, "cudaIpcOpenMemHandle(peer group)");
    g->peer[q] = (char*)p;
  }
  g->opened = true;
  return AMC_OK;
}

int amc_peer_sum(uint64_t h, const void* src, int64_t n, int32_t dtype, void* out, void* stream) {
  PeerGroup* g = group_get(h);
  if (!g || !g->opened) return fail(AMC_ERR_STATE, "amc_peer_sum: unknown or unopened group");
  if (!src || !out || n < 0 || (dtype != AMC_F32 && dtype != AMC_F64))
    return fail(AMC_ERR_INVALID, "amc_peer_sum: f32 or f64 device vectors");
  const int64_t esize = dtype == AMC_F32 ? 4 : 8;
  if (n * esize > g->max_elems * 8) return fail(AMC_ERR_INVALID, "amc_peer_sum: vector larger than the group's slots");
  if (fault_injected("launch")) return fail(AMC_ERR_INJECTED, "peer sum: injected launch failure (AMC_FAULT=launch)");
  cudaStream_t s = pick_stream(stream);
  const int64_t e = ++g->epoch;
  const int64_t slot_bytes = g->max_elems * 8;
  const int64_t parity_off = (int64_t)kFlagBytes + (e & 1) * g->world * slot_bytes;
  PushArgs pa;
  memset(&pa, 0, sizeof pa);
  pa.src = src; pa.n = n; pa.esize = (int32_t)esize; pa.world = g->world;
  pa.slot_off = parity_off + g->rank * slot_bytes;
  for (int q = 0; q < g->world; ++q) pa.peer[q] = g->peer[q];
  // 128-thread CTAs with few registers fit beside a resident tensor-core CTA
  // on the same SM, so the sum can overlap other work of the step
  const int blocks = (int)std::min<int64_t>(num_sms(), std::max<int64_t>(1, (n * esize / 16 + kDistThreads - 1) / kDistThreads));
  k_peer_push<<<blocks, kDistThreads, 0, s>>>(pa);
  AMC_CUDA(cudaGetLastError());
  SumArgs sa;
  memset(&sa, 0, sizeof sa);
  sa.out = out; sa.n = n; sa.dtype = dtype; sa.world = g->world; sa.rank = g->rank; sa.epoch = e;
  sa.slot_off0 = parity_off;
  sa.slot_stride = slot_bytes;
  sa.base = g->base;
  sa.flags_local = (volatile unsigned long long*)g->base;
  for (int q = 0; q < g->world; ++q) sa.peer[q] = g->peer[q];
  const int sblocks = (int)std::min<int64_t>(num_sms(), std::max<int64_t>(1, (n + kDistThreads - 1) / kDistThreads));
  k_peer_signal_sum<<<sblocks, kDistThreads, 0, s>>>(sa);
  AMC_CUDA(cudaGetLastError());
  return AMC_OK;
}

int amc_peer_group_destroy(uint64_t h) {
  PeerGroup* g = nullptr;
  {
    std::lock_guard<std::mutex> l(g_groups_mu);
    auto it = g_groups.find(h);
    if (it == g_groups.end()) return fail(AMC_ERR_INVALID, "amc_peer_group_destroy: unknown group");
    g = it->second;
    g_groups.erase(it);
  }
  cudaDeviceSynchronize();
  for (int q = 0; q < (int)g->peer.size(); ++q)
    if (q != g->rank && g->peer[q]) cudaIpcCloseMemHandle(g->peer[q]);
  cudaFree(g->base);
  delete g;
  return AMC_OK;
}

}  // extern "C"
