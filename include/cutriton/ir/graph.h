#pragma once

// Static-graph IR: Values (named tensor descriptions), Nodes (one operator
// each) and the Graph/Model that own them. API of the reference's
// include/cutriton/ir/graph.h:22-163.

#include <optional>
#include <string>
#include <unordered_map>
#include <utility>
#include <variant>
#include <vector>

#include "cutriton/core/tensor.h"

namespace cutriton {

using Attribute = std::variant<int64_t, double, bool, std::string,
                               std::vector<int64_t>, std::vector<double>>;

struct ValueDesc {
  std::string name;
  TensorDesc tensor;
  bool is_constant{false};
};

class Node {
 public:
  Node() = default;
  Node(std::string name, std::string op_type, std::vector<std::string> inputs,
       std::vector<std::string> outputs)
      : name_(std::move(name)), op_type_(std::move(op_type)),
        inputs_(std::move(inputs)), outputs_(std::move(outputs)) {}

  int id() const { return id_; }
  const std::string& name() const { return name_; }
  const std::string& op_type() const { return op_type_; }
  const std::vector<std::string>& inputs() const { return inputs_; }
  const std::vector<std::string>& outputs() const { return outputs_; }
  const std::unordered_map<std::string, Attribute>& attributes() const {
    return attributes_;
  }
  void set_name(std::string name) { name_ = std::move(name); }
  void set_op_type(std::string op_type) { op_type_ = std::move(op_type); }
  void set_inputs(std::vector<std::string> inputs) { inputs_ = std::move(inputs); }
  void set_outputs(std::vector<std::string> outputs) { outputs_ = std::move(outputs); }
  void SetAttribute(std::string key, Attribute value) {
    attributes_[std::move(key)] = std::move(value);
  }
  // Typed lookup; nullopt when missing or of another type.
  template <typename T>
  std::optional<T> GetAttribute(const std::string& key) const {
    const auto it = attributes_.find(key);
    if (it == attributes_.end()) return std::nullopt;
    if (const T* value = std::get_if<T>(&it->second)) return *value;
    return std::nullopt;
  }

 private:
  friend class Graph;
  void set_id(int id) { id_ = id; }

  int id_{-1};
  std::string name_;
  std::string op_type_;
  std::vector<std::string> inputs_;
  std::vector<std::string> outputs_;
  std::unordered_map<std::string, Attribute> attributes_;
};

class Graph {
 public:
  Status AddValue(ValueDesc value);
  Status AddInput(std::string name, TensorDesc desc);
  Status AddOutput(std::string name);
  Status AddNode(Node node);

  const std::vector<Node>& nodes() const { return nodes_; }
  std::vector<Node>& mutable_nodes() { return nodes_; }
  const std::unordered_map<std::string, ValueDesc>& values() const { return values_; }
  const std::vector<std::string>& inputs() const { return inputs_; }
  const std::vector<std::string>& outputs() const { return outputs_; }

  const ValueDesc* FindValue(const std::string& name) const;
  ValueDesc* MutableValue(const std::string& name);
  Status SetValueDesc(const std::string& name, TensorDesc desc);
  Status EnsureValue(std::string name, TensorDesc desc = {});
  // Kahn ordering; kInvalidArgument on a cycle.
  Status TopologicalSort();
  // Removes nodes by id and renumbers the rest densely.
  Status RemoveNodes(const std::vector<int>& node_ids);
  std::unordered_map<std::string, int> BuildProducerMap() const;
  std::unordered_map<std::string, std::vector<int>> BuildConsumerMap() const;

 private:
  void RenumberNodes();

  std::vector<Node> nodes_;
  std::unordered_map<std::string, ValueDesc> values_;
  std::vector<std::string> inputs_;
  std::vector<std::string> outputs_;
};

class Model {
 public:
  Graph& graph() { return graph_; }
  const Graph& graph() const { return graph_; }
  // Host-resident constant (weights); uploaded once per engine.
  Status AddConstant(std::string name, Tensor tensor);
  const std::unordered_map<std::string, Tensor>& constants() const { return constants_; }

 private:
  Graph graph_;
  std::unordered_map<std::string, Tensor> constants_;
};

std::vector<int64_t> GetIntListAttribute(const Node& node, const std::string& key,
                                         std::vector<int64_t> fallback);
int64_t GetIntAttribute(const Node& node, const std::string& key, int64_t fallback);

}  // namespace cutriton
