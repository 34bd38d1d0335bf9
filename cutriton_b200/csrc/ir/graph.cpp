// Graph / Model containers.
//
// The public surface is fixed by include/cutriton/ir/graph.h (the drop-in
// API). Internally:
//   * every name check goes through one helper, so all "empty name" failures
//     read the same way;
//   * the topological order is a depth-first post-order that visits nodes in
//     their current order and walks each node's producers first, so an order
//     that is already valid comes back unchanged; a node reached again while
//     it is still on the walk stack closes a cycle;
//   * node removal marks ids in a bitmap and compacts in place.

#include "cutriton/ir/graph.h"

#include <algorithm>
#include <utility>

#include "cutriton/core/buffer.h"

namespace cutriton {
namespace {

Status RequireName(const std::string& name, const char* what) {
  if (!name.empty()) return Status::OK();
  return Status::InvalidArgument(std::string(what) + ": the name is empty");
}

}  // namespace

Status Graph::AddValue(ValueDesc value) {
  CUTRITON_RETURN_IF_ERROR(RequireName(value.name, "Graph::AddValue"));
  auto slot = values_.try_emplace(value.name);
  if (!slot.second) return Status::AlreadyExists("Graph::AddValue: '" + value.name + "' is already defined");
  slot.first->second = std::move(value);
  return Status::OK();
}

Status Graph::AddInput(std::string name, TensorDesc desc) {
  CUTRITON_RETURN_IF_ERROR(RequireName(name, "Graph::AddInput"));
  // An input may name a value that a node already mentions: it then takes
  // the input's description.
  ValueDesc& value = values_[name];
  value.name = name;
  value.tensor = std::move(desc);
  inputs_.push_back(std::move(name));
  return Status::OK();
}

Status Graph::AddOutput(std::string name) {
  if (FindValue(name) == nullptr) {
    return Status::NotFound("Graph::AddOutput: no value named '" + name + "'");
  }
  outputs_.push_back(std::move(name));
  return Status::OK();
}

Status Graph::AddNode(Node node) {
  CUTRITON_RETURN_IF_ERROR(RequireName(node.name(), "Graph::AddNode"));
  if (node.op_type().empty()) {
    return Status::InvalidArgument("Graph::AddNode: node '" + node.name() + "' has no op_type");
  }
  // Values a node mentions come into existence with an empty description
  // (shape inference fills it in later).
  for (const auto* names : {&node.outputs(), &node.inputs()}) {
    for (const auto& name : *names) CUTRITON_RETURN_IF_ERROR(EnsureValue(name));
  }
  node.set_id(static_cast<int>(nodes_.size()));
  nodes_.push_back(std::move(node));
  return Status::OK();
}

const ValueDesc* Graph::FindValue(const std::string& name) const {
  const auto found = values_.find(name);
  return found != values_.end() ? &found->second : nullptr;
}

ValueDesc* Graph::MutableValue(const std::string& name) {
  return const_cast<ValueDesc*>(static_cast<const Graph*>(this)->FindValue(name));
}

Status Graph::SetValueDesc(const std::string& name, TensorDesc desc) {
  ValueDesc* value = MutableValue(name);
  if (value == nullptr) return Status::NotFound("Graph::SetValueDesc: no value named '" + name + "'");
  value->tensor = std::move(desc);
  return Status::OK();
}

Status Graph::EnsureValue(std::string name, TensorDesc desc) {
  CUTRITON_RETURN_IF_ERROR(RequireName(name, "Graph::EnsureValue"));
  auto slot = values_.try_emplace(name);
  if (slot.second) {
    slot.first->second.name = std::move(name);
    slot.first->second.tensor = std::move(desc);
  }
  return Status::OK();
}

std::unordered_map<std::string, int> Graph::BuildProducerMap() const {
  // A value written twice keeps its last writer.
  std::unordered_map<std::string, int> producer;
  for (const Node& node : nodes_) {
    for (const std::string& name : node.outputs()) producer[name] = node.id();
  }
  return producer;
}

std::unordered_map<std::string, std::vector<int>> Graph::BuildConsumerMap() const {
  std::unordered_map<std::string, std::vector<int>> readers;
  for (const Node& node : nodes_) {
    for (const std::string& name : node.inputs()) readers[name].push_back(node.id());
  }
  return readers;
}

Status Graph::TopologicalSort() {
  RenumberNodes();  // ids = positions, whatever a pass left behind
  const std::size_t count = nodes_.size();
  const auto producer = BuildProducerMap();
  // Producers of each node's inputs, in input order (a node reading its own
  // output does not depend on itself).
  std::vector<std::vector<int>> needs(count);
  for (const Node& node : nodes_) {
    for (const std::string& name : node.inputs()) {
      const auto found = producer.find(name);
      if (found != producer.end() && found->second != node.id()) needs[node.id()].push_back(found->second);
    }
  }

  enum : char { kUnseen = 0, kOnStack = 1, kPlaced = 2 };
  std::vector<char> state(count, kUnseen);
  std::vector<int> order;
  order.reserve(count);
  // Explicit stack of (node, next dependency to look at).
  std::vector<std::pair<int, std::size_t>> walk;
  for (std::size_t root = 0; root < count; ++root) {
    if (state[root] != kUnseen) continue;
    walk.emplace_back(static_cast<int>(root), 0);
    state[root] = kOnStack;
    while (!walk.empty()) {
      auto& [id, next] = walk.back();
      if (next < needs[id].size()) {
        const int dep = needs[id][next++];
        if (state[dep] == kOnStack) {
          return Status::InvalidArgument("Graph::TopologicalSort: node '" + nodes_[dep].name() +
                                         "' depends on itself through a cycle");
        }
        if (state[dep] == kUnseen) {
          state[dep] = kOnStack;
          walk.emplace_back(dep, 0);
        }
        continue;
      }
      state[id] = kPlaced;
      order.push_back(id);
      walk.pop_back();
    }
  }

  std::vector<Node> sorted;
  sorted.reserve(count);
  for (int id : order) sorted.push_back(std::move(nodes_[id]));
  nodes_ = std::move(sorted);
  RenumberNodes();
  return Status::OK();
}

Status Graph::RemoveNodes(const std::vector<int>& node_ids) {
  std::vector<char> doomed(nodes_.size(), 0);
  for (int id : node_ids) {
    if (id >= 0 && static_cast<std::size_t>(id) < doomed.size()) doomed[id] = 1;
  }
  // Ids are dense after every renumbering; a node appended through
  // mutable_nodes() without one is never matched.
  const auto marked = [&](const Node& node) {
    return node.id() >= 0 && static_cast<std::size_t>(node.id()) < doomed.size() && doomed[node.id()] != 0;
  };
  nodes_.erase(std::remove_if(nodes_.begin(), nodes_.end(), marked), nodes_.end());
  RenumberNodes();
  return Status::OK();
}

void Graph::RenumberNodes() {
  int next = 0;
  for (Node& node : nodes_) node.set_id(next++);
}

std::vector<int64_t> GetIntListAttribute(const Node& node, const std::string& key,
                                         std::vector<int64_t> fallback) {
  auto value = node.GetAttribute<std::vector<int64_t>>(key);
  return value ? std::move(*value) : std::move(fallback);
}

int64_t GetIntAttribute(const Node& node, const std::string& key, int64_t fallback) {
  return node.GetAttribute<int64_t>(key).value_or(fallback);
}

Status Model::AddConstant(std::string name, Tensor tensor) {
  CUTRITON_RETURN_IF_ERROR(RequireName(name, "Model::AddConstant"));
  CUTRITON_RETURN_IF_ERROR(tensor.desc().Validate());
  const std::string where = "Model::AddConstant('" + name + "'): ";
  if (!tensor.defined() || tensor.buffer()->empty()) return Status::InvalidArgument(where + "no data");
  if (tensor.buffer()->device_type() != DeviceType::kCPU || tensor.desc().device_type != DeviceType::kCPU) {
    return Status::InvalidArgument(where + "constants are host tensors");
  }
  const std::size_t capacity = tensor.buffer()->size_bytes();
  const std::size_t needed = tensor.desc().ByteSize();
  if (tensor.byte_offset() > capacity || needed > capacity - tensor.byte_offset()) {
    return Status::InvalidArgument(where + "the buffer holds fewer bytes than the description needs");
  }
  const ValueDesc* existing = graph_.FindValue(name);
  if (constants_.count(name) != 0 || (existing != nullptr && existing->is_constant)) {
    return Status::AlreadyExists(where + "already defined");
  }
  // A value the graph already mentions (e.g. a node input declared before
  // the weights) becomes the constant.
  if (existing == nullptr) {
    CUTRITON_RETURN_IF_ERROR(graph_.AddValue(ValueDesc{name, tensor.desc(), true}));
  } else {
    ValueDesc* value = graph_.MutableValue(name);
    value->tensor = tensor.desc();
    value->is_constant = true;
  }
  constants_.emplace(std::move(name), std::move(tensor));
  return Status::OK();
}

}  // namespace cutriton
