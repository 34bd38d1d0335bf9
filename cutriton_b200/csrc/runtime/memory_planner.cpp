// Single-workspace memory planner.
//
// Same policy as the reference planner (src/runtime/memory_planner.cpp:29-169):
// graph inputs/outputs and constants are external; every other value gets a
// 256-byte aligned slot; a slot is freed once the value's last consumer ran
// and reused best-fit (smallest free block that fits, split when larger);
// Flatten outputs alias their input and extend its lifetime.

#include "cutriton/runtime/memory_planner.h"

#include <algorithm>
#include <unordered_map>
#include <unordered_set>

namespace cutriton {
namespace {

constexpr std::size_t kAlignment = 256;

std::size_t AlignUp(std::size_t bytes) { return (bytes + kAlignment - 1) / kAlignment * kAlignment; }

struct Block {
  std::size_t offset;
  std::size_t size;
};

}  // namespace

Status MemoryPlanner::Plan(const Graph& graph, MemoryPlan* plan) const {
  if (plan == nullptr) return Status::InvalidArgument("MemoryPlan output pointer is null");
  *plan = MemoryPlan{};
  std::unordered_set<std::string> external(graph.inputs().begin(), graph.inputs().end());
  external.insert(graph.outputs().begin(), graph.outputs().end());

  std::unordered_map<std::string, std::string> alias_source;
  for (const auto& node : graph.nodes()) {
    if (node.op_type() == "Flatten" && node.inputs().size() == 1 && node.outputs().size() == 1) {
      alias_source[node.outputs()[0]] = node.inputs()[0];
    }
  }

  // Index of the last node that reads each value (outputs: past the end).
  std::unordered_map<std::string, int> last_read;
  const int node_count = static_cast<int>(graph.nodes().size());
  for (int i = 0; i < node_count; ++i) {
    const Node& node = graph.nodes()[static_cast<std::size_t>(i)];
    for (const auto& v : node.inputs()) last_read[v] = i;
    for (const auto& v : node.outputs()) last_read.emplace(v, i);
  }
  for (const auto& v : graph.outputs()) last_read[v] = node_count;
  for (const auto& entry : alias_source) {
    const auto alias = last_read.find(entry.first);
    if (alias != last_read.end()) {
      int& source = last_read[entry.second];
      source = std::max(source, alias->second);
    }
  }

  std::vector<Block> free_list;
  std::vector<std::pair<std::string, Block>> live;
  std::unordered_map<std::string, Allocation> placed;
  std::size_t high_water = 0;

  for (int i = 0; i < node_count; ++i) {
    // Retire values whose last reader ran before this node.
    for (auto it = live.begin(); it != live.end();) {
      const auto use = last_read.find(it->first);
      if (use != last_read.end() && use->second < i) {
        free_list.push_back(it->second);
        it = live.erase(it);
      } else {
        ++it;
      }
    }
    const Node& node = graph.nodes()[static_cast<std::size_t>(i)];
    for (const auto& name : node.outputs()) {
      if (external.count(name) != 0) continue;
      const auto alias = alias_source.find(name);
      if (alias != alias_source.end()) {
        const auto source = placed.find(alias->second);
        Allocation a;
        if (source != placed.end()) {
          a = source->second;
        } else {
          if (external.count(alias->second) == 0) {
            return Status::Internal("Flatten alias source has no allocation: " + alias->second);
          }
          const ValueDesc* src = graph.FindValue(alias->second);
          if (src == nullptr) return Status::Internal("Flatten alias source is unknown: " + alias->second);
          a.size_bytes = src->tensor.ByteSize();
        }
        a.value_name = name;
        a.alias_of = alias->second;
        a.reused = true;
        const ValueDesc* value = graph.FindValue(name);
        if (value == nullptr || value->tensor.ByteSize() != a.size_bytes) {
          return Status::ShapeError("Flatten alias changes the tensor byte size: " + name);
        }
        plan->allocations.push_back(a);
        placed.emplace(name, a);
        continue;
      }
      const ValueDesc* value = graph.FindValue(name);
      if (value == nullptr || value->is_constant) continue;
      const std::size_t bytes = value->tensor.ByteSize();
      if (bytes == 0) return Status::ShapeError("cannot plan memory for a dynamically sized value: " + name);
      const std::size_t reserved = AlignUp(bytes);
      auto best = free_list.end();
      for (auto it = free_list.begin(); it != free_list.end(); ++it) {
        if (it->size >= reserved && (best == free_list.end() || it->size < best->size)) best = it;
      }
      Allocation a;
      a.value_name = name;
      a.size_bytes = bytes;
      if (best != free_list.end()) {
        a.offset = best->offset;
        a.reused = true;
        if (best->size > reserved) {
          best->offset += reserved;
          best->size -= reserved;
        } else {
          free_list.erase(best);
        }
      } else {
        a.offset = AlignUp(high_water);
        high_water = a.offset + reserved;
      }
      plan->allocations.push_back(a);
      placed.emplace(name, a);
      live.push_back({name, Block{a.offset, reserved}});
    }
  }
  plan->workspace_size_bytes = AlignUp(high_water);
  return Status::OK();
}

}  // namespace cutriton
