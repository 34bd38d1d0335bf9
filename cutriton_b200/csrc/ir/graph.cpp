#include "cutriton/ir/graph.h"

#include <functional>
#include <queue>
#include <unordered_set>

#include "cutriton/core/buffer.h"

namespace cutriton {

Status Graph::AddValue(ValueDesc value) {
  if (value.name.empty()) return Status::InvalidArgument("value name must not be empty");
  const std::string key = value.name;
  if (!values_.emplace(key, std::move(value)).second) {
    return Status::AlreadyExists("value already exists: " + key);
  }
  return Status::OK();
}

Status Graph::AddInput(std::string name, TensorDesc desc) {
  if (name.empty()) return Status::InvalidArgument("input name must not be empty");
  if (values_.count(name) == 0) {
    CUTRITON_RETURN_IF_ERROR(AddValue(ValueDesc{name, std::move(desc), false}));
  } else {
    CUTRITON_RETURN_IF_ERROR(SetValueDesc(name, std::move(desc)));
  }
  inputs_.push_back(std::move(name));
  return Status::OK();
}

Status Graph::AddOutput(std::string name) {
  if (values_.count(name) == 0) return Status::NotFound("graph output value is undefined: " + name);
  outputs_.push_back(std::move(name));
  return Status::OK();
}

Status Graph::AddNode(Node node) {
  if (node.name().empty()) return Status::InvalidArgument("node name must not be empty");
  if (node.op_type().empty()) return Status::InvalidArgument("node op_type must not be empty");
  for (const auto& name : node.outputs()) CUTRITON_RETURN_IF_ERROR(EnsureValue(name));
  for (const auto& name : node.inputs()) CUTRITON_RETURN_IF_ERROR(EnsureValue(name));
  node.set_id(static_cast<int>(nodes_.size()));
  nodes_.push_back(std::move(node));
  return Status::OK();
}

const ValueDesc* Graph::FindValue(const std::string& name) const {
  const auto it = values_.find(name);
  return it == values_.end() ? nullptr : &it->second;
}

ValueDesc* Graph::MutableValue(const std::string& name) {
  const auto it = values_.find(name);
  return it == values_.end() ? nullptr : &it->second;
}

Status Graph::SetValueDesc(const std::string& name, TensorDesc desc) {
  ValueDesc* value = MutableValue(name);
  if (value == nullptr) return Status::NotFound("value is undefined: " + name);
  value->tensor = std::move(desc);
  return Status::OK();
}

Status Graph::EnsureValue(std::string name, TensorDesc desc) {
  if (name.empty()) return Status::InvalidArgument("value name must not be empty");
  if (values_.count(name) == 0) {
    ValueDesc value{name, std::move(desc), false};
    values_.emplace(std::move(name), std::move(value));
  }
  return Status::OK();
}

std::unordered_map<std::string, int> Graph::BuildProducerMap() const {
  std::unordered_map<std::string, int> producers;
  for (const auto& node : nodes_) {
    for (const auto& output : node.outputs()) producers[output] = node.id();
  }
  return producers;
}

std::unordered_map<std::string, std::vector<int>> Graph::BuildConsumerMap() const {
  std::unordered_map<std::string, std::vector<int>> consumers;
  for (const auto& node : nodes_) {
    for (const auto& input : node.inputs()) consumers[input].push_back(node.id());
  }
  return consumers;
}

// Stable Kahn ordering: among ready nodes the one added earliest runs first,
// so an already valid order is kept unchanged.
Status Graph::TopologicalSort() {
  const auto producers = BuildProducerMap();
  const std::size_t count = nodes_.size();
  std::vector<int> pending(count, 0);
  std::vector<std::vector<int>> successors(count);
  for (const auto& node : nodes_) {
    std::unordered_set<int> deps;
    for (const auto& input : node.inputs()) {
      const auto it = producers.find(input);
      if (it != producers.end() && it->second != node.id()) deps.insert(it->second);
    }
    pending[node.id()] = static_cast<int>(deps.size());
    for (int dep : deps) successors[dep].push_back(node.id());
  }
  std::priority_queue<int, std::vector<int>, std::greater<int>> ready;
  for (std::size_t i = 0; i < count; ++i) {
    if (pending[i] == 0) ready.push(static_cast<int>(i));
  }
  std::vector<Node> ordered;
  ordered.reserve(count);
  while (!ready.empty()) {
    const int id = ready.top();
    ready.pop();
    ordered.push_back(nodes_[id]);
    for (int next : successors[id]) {
      if (--pending[next] == 0) ready.push(next);
    }
  }
  if (ordered.size() != count) return Status::InvalidArgument("graph contains a cycle");
  nodes_ = std::move(ordered);
  RenumberNodes();
  return Status::OK();
}

Status Graph::RemoveNodes(const std::vector<int>& node_ids) {
  const std::unordered_set<int> doomed(node_ids.begin(), node_ids.end());
  std::vector<Node> kept;
  kept.reserve(nodes_.size());
  for (auto& node : nodes_) {
    if (doomed.count(node.id()) == 0) kept.push_back(std::move(node));
  }
  nodes_ = std::move(kept);
  RenumberNodes();
  return Status::OK();
}

void Graph::RenumberNodes() {
  for (std::size_t i = 0; i < nodes_.size(); ++i) nodes_[i].set_id(static_cast<int>(i));
}

std::vector<int64_t> GetIntListAttribute(const Node& node, const std::string& key,
                                         std::vector<int64_t> fallback) {
  if (auto value = node.GetAttribute<std::vector<int64_t>>(key)) return *value;
  return fallback;
}

int64_t GetIntAttribute(const Node& node, const std::string& key, int64_t fallback) {
  if (auto value = node.GetAttribute<int64_t>(key)) return *value;
  return fallback;
}

Status Model::AddConstant(std::string name, Tensor tensor) {
  if (name.empty()) return Status::InvalidArgument("constant name must not be empty");
  CUTRITON_RETURN_IF_ERROR(tensor.desc().Validate());
  if (!tensor.defined() || tensor.buffer()->empty()) {
    return Status::InvalidArgument("constant tensor has no buffer: " + name);
  }
  if (tensor.buffer()->device_type() != DeviceType::kCPU ||
      tensor.desc().device_type != DeviceType::kCPU) {
    return Status::InvalidArgument("model constants must live in host memory: " + name);
  }
  const std::size_t capacity = tensor.buffer()->size_bytes();
  if (tensor.byte_offset() > capacity ||
      tensor.desc().ByteSize() > capacity - tensor.byte_offset()) {
    return Status::InvalidArgument("constant buffer is too small: " + name);
  }
  if (constants_.count(name) != 0) return Status::AlreadyExists("constant already exists: " + name);
  if (const ValueDesc* existing = graph_.FindValue(name)) {
    if (existing->is_constant) return Status::AlreadyExists("constant already exists: " + name);
    CUTRITON_RETURN_IF_ERROR(graph_.SetValueDesc(name, tensor.desc()));
    graph_.MutableValue(name)->is_constant = true;
  } else {
    CUTRITON_RETURN_IF_ERROR(graph_.AddValue(ValueDesc{name, tensor.desc(), true}));
  }
  constants_.emplace(std::move(name), std::move(tensor));
  return Status::OK();
}

}  // namespace cutriton
