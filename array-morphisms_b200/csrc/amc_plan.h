// Plans and contexts shared between the planner and the context arena.
#pragma once

#include <functional>
#include <vector>

#include "amc_internal.h"

namespace amc {

struct Plan {
  void* ctx = nullptr;                       // owning context (realize/ctx) or null
  std::vector<std::function<int(cudaStream_t)>> steps;
  std::vector<uint64_t> slots;               // buffers this plan allocated (one ref each)
  std::vector<uint64_t> held;                // leaf buffers kept alive
  std::vector<void*> dev_small;              // small device tables (stack/concat operands)
  std::vector<int32_t> slot_alloc_ids;       // context allocation id of each slot
  amc_view result{};                         // results[0]
  std::vector<amc_view> results;             // one per root (one reference each)
  bool result_owned = false;
  int32_t ctx_first_id = 0;                  // replay mode: the context allocation ids
  int32_t ctx_ids = 0;                       // this plan took, [first, first + ids)
  bool ctx_replay = false;
  int32_t launches = 0;
  int64_t bytes = 0;
  bool used_fir = false;
  cudaGraphExec_t graph_exec = nullptr;

  int add_slot(int32_t dtype, int64_t n, const std::vector<uint64_t>& reads, uint64_t* h);
  ~Plan();
};

// Context allocation hook: trace mode allocates and records, replay mode
// hands out arena sub-buffers by allocation counter.
int ctx_alloc(void* ctx, int32_t dtype, int64_t n, const std::vector<uint64_t>& reads, uint64_t* h);
// The context's mode (0 trace, 1 replay) and its replay allocation counter.
int ctx_mode(void* ctx);
int32_t ctx_counter(void* ctx);

int plan_create(void* ctx, const amc_node* nodes, int32_t n, uint64_t* out);
Plan* plan_get(uint64_t h);
int plan_execute(Plan* p, cudaStream_t s);

}  // namespace amc
