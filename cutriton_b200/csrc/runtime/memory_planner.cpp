// Workspace planner for the intermediate tensors of one graph.
//
// Contract (include/cutriton/runtime/memory_planner.h): graph inputs, graph
// outputs and constants live outside the workspace; every other value gets a
// 256-byte aligned range that no value alive at the same time overlaps; a
// Flatten output is a view of its input (same range, and the input stays
// alive as long as the view is read).
//
// Method: an offline interval plan rather than a free list walked in node
// order.
//   1. Lifetimes. A value is alive from the node that writes it to the last
//      node that reads it, inclusive (a node's inputs and outputs never
//      share memory); a Flatten view extends its source's lifetime.
//   2. Placement, largest value first (ties: earlier definition first): each
//      value takes the lowest aligned offset that overlaps no placed value
//      whose lifetime intersects its own. Sorting by size keeps big tensors
//      packed at the bottom and lets small short-lived ones fill the gaps.
//   3. Views take their source's range. Allocations are reported in
//      definition order; `reused` marks a range that an earlier value with a
//      disjoint lifetime also occupied.

#include "cutriton/runtime/memory_planner.h"

#include <algorithm>
#include <unordered_map>
#include <unordered_set>

namespace cutriton {
namespace {

constexpr std::size_t kAlign = 256;

std::size_t RoundUp(std::size_t bytes) { return (bytes + kAlign - 1) / kAlign * kAlign; }

struct Interval {
  std::string name;
  int first{0};           // node that writes the value
  int last{0};            // last node that reads it (>= first)
  std::size_t bytes{0};   // tensor bytes
  std::size_t span{0};    // bytes rounded up to the alignment
  std::size_t offset{0};
  std::string view_of;    // non-empty for a Flatten view
  std::size_t order{0};   // definition order
};

bool Overlap(std::size_t a, std::size_t a_len, std::size_t b, std::size_t b_len) {
  return a < b + b_len && b < a + a_len;
}

}  // namespace

Status MemoryPlanner::Plan(const Graph& graph, MemoryPlan* plan) const {
  if (plan == nullptr) return Status::InvalidArgument("MemoryPlanner::Plan: no MemoryPlan to write");
  *plan = MemoryPlan{};
  const auto& nodes = graph.nodes();
  const int end_of_graph = static_cast<int>(nodes.size());

  std::unordered_set<std::string> outside(graph.inputs().begin(), graph.inputs().end());
  for (const auto& name : graph.outputs()) outside.insert(name);

  // ---- 1. lifetimes ---------------------------------------------------------
  std::vector<Interval> values;
  std::unordered_map<std::string, std::size_t> index;  // name -> position in `values`
  std::unordered_map<std::string, int> last_read;
  for (int at = 0; at < end_of_graph; ++at) {
    for (const auto& name : nodes[at].inputs()) last_read[name] = at;
  }
  for (const auto& name : graph.outputs()) last_read[name] = end_of_graph;

  for (int at = 0; at < end_of_graph; ++at) {
    const Node& node = nodes[at];
    const bool is_view = node.op_type() == "Flatten" && node.inputs().size() == 1 && node.outputs().size() == 1;
    for (const auto& name : node.outputs()) {
      if (outside.count(name) != 0 || index.count(name) != 0) continue;
      const ValueDesc* desc = graph.FindValue(name);
      if (desc == nullptr || (desc->is_constant && !is_view)) continue;
      Interval v;
      v.name = name;
      v.first = at;
      const auto read = last_read.find(name);
      v.last = read == last_read.end() ? at : std::max(at, read->second);
      v.bytes = desc->tensor.ByteSize();
      v.order = values.size();
      if (is_view) {
        v.view_of = node.inputs()[0];
      } else if (v.bytes == 0) {
        return Status::ShapeError("MemoryPlanner::Plan: '" + name + "' has no static size (unresolved shape)");
      }
      v.span = RoundUp(v.bytes);
      index.emplace(name, values.size());
      values.push_back(std::move(v));
    }
  }
  // Views keep their source alive. A view is defined after its source, so
  // walking back to front carries the lifetime of a chain of views down to
  // the planned value at its root.
  for (auto v = values.rbegin(); v != values.rend(); ++v) {
    if (v->view_of.empty()) continue;
    const auto source = index.find(v->view_of);
    if (source != index.end()) {
      Interval& s = values[source->second];
      s.last = std::max(s.last, v->last);
    }
  }
  for (Interval& v : values) {
    if (v.view_of.empty()) continue;
    const auto source = index.find(v.view_of);
    if (source != index.end()) {
      const Interval& s = values[source->second];
      if (s.bytes != v.bytes) {
        return Status::ShapeError("MemoryPlanner::Plan: Flatten view '" + v.name + "' has " +
                                  std::to_string(v.bytes) + " bytes, its source " + std::to_string(s.bytes));
      }
      continue;
    }
    // A view of a graph input lives outside the workspace like its source.
    if (outside.count(v.view_of) == 0) {
      return Status::Internal("MemoryPlanner::Plan: the source of Flatten view '" + v.name +
                              "' is neither planned nor external: " + v.view_of);
    }
    const ValueDesc* src = graph.FindValue(v.view_of);
    if (src == nullptr || src->tensor.ByteSize() != v.bytes) {
      return Status::ShapeError("MemoryPlanner::Plan: Flatten view '" + v.name + "' changes the byte size");
    }
  }

  // ---- 2. placement, largest first --------------------------------------------
  std::vector<std::size_t> by_size;
  for (std::size_t i = 0; i < values.size(); ++i) {
    if (values[i].view_of.empty()) by_size.push_back(i);
  }
  std::stable_sort(by_size.begin(), by_size.end(),
                   [&](std::size_t a, std::size_t b) { return values[a].span > values[b].span; });
  std::vector<std::size_t> placed;
  std::size_t top = 0;
  for (std::size_t i : by_size) {
    Interval& v = values[i];
    // Ranges taken by placed values alive at the same time, sorted by offset.
    std::vector<std::pair<std::size_t, std::size_t>> busy;
    for (std::size_t j : placed) {
      const Interval& u = values[j];
      if (u.first <= v.last && v.first <= u.last) busy.emplace_back(u.offset, u.span);
    }
    std::sort(busy.begin(), busy.end());
    std::size_t candidate = 0;
    for (const auto& range : busy) {
      if (Overlap(candidate, v.span, range.first, range.second)) {
        candidate = std::max(candidate, RoundUp(range.first + range.second));
      }
    }
    v.offset = candidate;
    top = std::max(top, candidate + v.span);
    placed.push_back(i);
  }

  // ---- 3. report -----------------------------------------------------------------
  for (const Interval& v : values) {
    Allocation a;
    a.value_name = v.name;
    a.size_bytes = v.bytes;
    if (!v.view_of.empty()) {
      // Offset of the planned value at the root of the chain of views (0
      // for a view of an external value, which the engine binds directly).
      std::size_t offset = 0;
      for (auto at = index.find(v.view_of); at != index.end(); at = index.find(values[at->second].view_of)) {
        offset = values[at->second].offset;
        if (values[at->second].view_of.empty()) break;
      }
      a.offset = offset;
      a.alias_of = v.view_of;
      a.reused = true;
      plan->allocations.push_back(std::move(a));
      continue;
    }
    a.offset = v.offset;
    // Reused: an earlier-defined value with a disjoint lifetime sat here.
    for (const Interval& u : values) {
      if (u.order >= v.order) break;
      if (!u.view_of.empty()) continue;
      if (Overlap(u.offset, u.span, v.offset, v.span) && !(u.first <= v.last && v.first <= u.last)) {
        a.reused = true;
        break;
      }
    }
    plan->allocations.push_back(std::move(a));
  }
  plan->workspace_size_bytes = RoundUp(top);
  return Status::OK();
}

}  // namespace cutriton
