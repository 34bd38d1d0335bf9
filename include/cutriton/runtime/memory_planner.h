#pragma once

// Single-workspace planner for intermediate tensors (API of the reference's
// include/cutriton/runtime/memory_planner.h:13-29): 256-byte aligned slots,
// best-fit reuse once a value's last consumer has run, Flatten outputs alias
// their input.

#include <cstddef>
#include <string>
#include <vector>

#include "cutriton/core/status.h"
#include "cutriton/ir/graph.h"

namespace cutriton {

struct Allocation {
  std::string value_name;
  std::size_t size_bytes{0};
  std::size_t offset{0};
  bool reused{false};
  std::string alias_of;
};

struct MemoryPlan {
  std::size_t workspace_size_bytes{0};
  std::vector<Allocation> allocations;
};

class MemoryPlanner {
 public:
  Status Plan(const Graph& graph, MemoryPlan* plan) const;
};

}  // namespace cutriton
