// Graph passes, builtin op schemas and shape inference.
//
// Behaviour follows the reference pipeline (src/ir/pass.cpp:549-684): the
// same op set, arities, shape rules and fusion patterns, so graphs built for
// the reference engine compile to the same fused plan here. One pattern is
// added: FusedConvBatchNorm -> AddRelu  =>  FusedConvBatchNormAddRelu (the
// ResNet bottleneck tail), which keeps an unfused candidate for the tuner.

#include "cutriton/ir/pass.h"

#include <algorithm>
#include <unordered_set>

#include "cutriton/ir/op_schema.h"

namespace cutriton {
namespace {

bool IsGraphOutput(const Graph& graph, const std::string& name) {
  return std::find(graph.outputs().begin(), graph.outputs().end(), name) != graph.outputs().end();
}

int64_t DimProduct(const std::vector<int64_t>& dims, std::size_t begin, std::size_t end) {
  int64_t product = 1;
  for (std::size_t i = begin; i < end; ++i) {
    if (dims[i] <= 0) return 0;
    product *= dims[i];
  }
  return product;
}

TensorDesc Derived(const TensorDesc& like, std::vector<int64_t> shape, std::string layout) {
  return TensorDesc(std::move(shape), like.dtype, like.device_type, like.device_id,
                    std::move(layout));
}

// ---- shape inference -------------------------------------------------------

Status InferLikeFirstInput(Graph* graph, const Node& node) {
  const ValueDesc* first = node.inputs().empty() ? nullptr : graph->FindValue(node.inputs()[0]);
  if (first == nullptr || first->tensor.dtype == DataType::kUnknown) {
    return Status::ShapeError("cannot infer the shape of node " + node.name());
  }
  for (const auto& output : node.outputs()) {
    CUTRITON_RETURN_IF_ERROR(graph->SetValueDesc(output, first->tensor));
  }
  return Status::OK();
}

Status InferBinary(Graph* graph, const Node& node) {
  if (node.inputs().size() != 2 || node.outputs().size() != 1) {
    return Status::ShapeError(node.op_type() + " expects two inputs and one output");
  }
  const ValueDesc* a = graph->FindValue(node.inputs()[0]);
  const ValueDesc* b = graph->FindValue(node.inputs()[1]);
  if (a == nullptr || b == nullptr) return Status::ShapeError(node.op_type() + " references an unknown tensor");
  if (a->tensor.shape != b->tensor.shape || a->tensor.dtype != b->tensor.dtype ||
      a->tensor.layout != b->tensor.layout) {
    return Status::ShapeError(node.op_type() + " inputs must have identical descriptions");
  }
  return graph->SetValueDesc(node.outputs()[0], a->tensor);
}

Status InferConv(Graph* graph, const Node& node) {
  if (node.inputs().size() < 2 || node.outputs().empty()) {
    return Status::ShapeError("convolution needs input, weight and output");
  }
  const ValueDesc* x = graph->FindValue(node.inputs()[0]);
  const ValueDesc* w = graph->FindValue(node.inputs()[1]);
  if (x == nullptr || w == nullptr) return Status::ShapeError("convolution references an unknown tensor");
  const auto& xs = x->tensor.shape;
  const auto& ws = w->tensor.shape;
  if (xs.size() != 4 || ws.size() != 4) return Status::ShapeError("convolution expects NCHW input and OIHW weight");
  const auto strides = GetIntListAttribute(node, "strides", {1, 1});
  const auto pads = GetIntListAttribute(node, "pads", {0, 0, 0, 0});
  const auto dilations = GetIntListAttribute(node, "dilations", {1, 1});
  if (strides.size() != 2 || pads.size() != 4 || dilations.size() != 2) {
    return Status::ShapeError("convolution attributes must be strides[2], pads[4], dilations[2]");
  }
  const int64_t oh = (xs[2] + pads[0] + pads[2] - dilations[0] * (ws[2] - 1) - 1) / strides[0] + 1;
  const int64_t ow = (xs[3] + pads[1] + pads[3] - dilations[1] * (ws[3] - 1) - 1) / strides[1] + 1;
  TensorDesc out = Derived(x->tensor, {xs[0], ws[0], oh, ow}, x->tensor.layout);
  CUTRITON_RETURN_IF_ERROR(out.Validate());
  return graph->SetValueDesc(node.outputs()[0], std::move(out));
}

Status InferPool(Graph* graph, const Node& node) {
  const ValueDesc* x = graph->FindValue(node.inputs().front());
  if (x == nullptr || x->tensor.shape.size() != 4) return Status::ShapeError("pooling expects an NCHW input");
  const auto kernel = GetIntListAttribute(node, "kernel_shape", {1, 1});
  const auto strides = GetIntListAttribute(node, "strides", kernel);
  const auto pads = GetIntListAttribute(node, "pads", {0, 0, 0, 0});
  const auto dilations = GetIntListAttribute(node, "dilations", {1, 1});
  if (kernel.size() != 2 || strides.size() != 2 || pads.size() != 4 || dilations.size() != 2) {
    return Status::ShapeError("pooling attributes must be kernel_shape[2], strides[2], pads[4], dilations[2]");
  }
  const auto& s = x->tensor.shape;
  const int64_t span_h = dilations[0] * (kernel[0] - 1) + 1;
  const int64_t span_w = dilations[1] * (kernel[1] - 1) + 1;
  const int64_t oh = (s[2] + pads[0] + pads[2] - span_h) / strides[0] + 1;
  const int64_t ow = (s[3] + pads[1] + pads[3] - span_w) / strides[1] + 1;
  TensorDesc out = Derived(x->tensor, {s[0], s[1], oh, ow}, x->tensor.layout);
  CUTRITON_RETURN_IF_ERROR(out.Validate());
  return graph->SetValueDesc(node.outputs()[0], std::move(out));
}

Status InferGlobalAveragePool(Graph* graph, const Node& node) {
  const ValueDesc* x = graph->FindValue(node.inputs().front());
  if (x == nullptr || x->tensor.shape.size() != 4) {
    return Status::ShapeError("GlobalAveragePool expects an NCHW input");
  }
  const auto& s = x->tensor.shape;
  return graph->SetValueDesc(node.outputs()[0], Derived(x->tensor, {s[0], s[1], 1, 1}, x->tensor.layout));
}

Status InferFlatten(Graph* graph, const Node& node) {
  const ValueDesc* x = graph->FindValue(node.inputs().front());
  if (x == nullptr || x->tensor.shape.empty()) return Status::ShapeError("Flatten needs a known input shape");
  const auto& s = x->tensor.shape;
  int64_t axis = GetIntAttribute(node, "axis", 1);
  if (axis < 0) axis += static_cast<int64_t>(s.size());
  if (axis < 0 || axis > static_cast<int64_t>(s.size())) return Status::ShapeError("Flatten axis exceeds the input rank");
  const auto split = static_cast<std::size_t>(axis);
  TensorDesc out = Derived(x->tensor, {DimProduct(s, 0, split), DimProduct(s, split, s.size())}, "");
  CUTRITON_RETURN_IF_ERROR(out.Validate());
  return graph->SetValueDesc(node.outputs()[0], std::move(out));
}

Status InferGemm(Graph* graph, const Node& node) {
  if (node.inputs().size() < 2) return Status::ShapeError("Gemm expects two inputs");
  const ValueDesc* a = graph->FindValue(node.inputs()[0]);
  const ValueDesc* b = graph->FindValue(node.inputs()[1]);
  if (a == nullptr || b == nullptr || a->tensor.shape.size() != 2 || b->tensor.shape.size() != 2) {
    return Status::ShapeError("Gemm expects rank-2 inputs");
  }
  if (a->tensor.dtype != b->tensor.dtype) return Status::ShapeError("Gemm inputs must have the same dtype");
  const bool ta = GetIntAttribute(node, "transA", 0) != 0;
  const bool tb = GetIntAttribute(node, "transB", 0) != 0;
  const auto& as = a->tensor.shape;
  const auto& bs = b->tensor.shape;
  const int64_t m = ta ? as[1] : as[0];
  const int64_t ka = ta ? as[0] : as[1];
  const int64_t kb = tb ? bs[1] : bs[0];
  const int64_t n = tb ? bs[0] : bs[1];
  if (ka != kb) return Status::ShapeError("Gemm inner dimensions do not match");
  if (node.inputs().size() == 3) {
    const ValueDesc* bias = graph->FindValue(node.inputs()[2]);
    if (bias == nullptr || bias->tensor.dtype != a->tensor.dtype ||
        (bias->tensor.shape != std::vector<int64_t>{n} &&
         bias->tensor.shape != std::vector<int64_t>{m, n})) {
      return Status::ShapeError("Gemm bias must be [N] or [M,N]");
    }
  }
  TensorDesc out = Derived(a->tensor, {m, n}, "");
  CUTRITON_RETURN_IF_ERROR(out.Validate());
  return graph->SetValueDesc(node.outputs()[0], std::move(out));
}

Status CheckNormParams(const Graph& graph, const std::string& x_name,
                       const std::string& scale_name, const std::string* bias_name,
                       int64_t axis) {
  const ValueDesc* x = graph.FindValue(x_name);
  const ValueDesc* scale = graph.FindValue(scale_name);
  if (x == nullptr || scale == nullptr || x->tensor.shape.empty() ||
      scale->tensor.shape != std::vector<int64_t>{x->tensor.shape.back()} ||
      x->tensor.dtype != scale->tensor.dtype) {
    return Status::ShapeError("LayerNormalization scale must match the last dimension");
  }
  if (bias_name != nullptr) {
    const ValueDesc* bias = graph.FindValue(*bias_name);
    if (bias == nullptr || bias->tensor.shape != scale->tensor.shape ||
        bias->tensor.dtype != x->tensor.dtype) {
      return Status::ShapeError("LayerNormalization bias must match scale");
    }
  }
  if (axis != -1 && axis != static_cast<int64_t>(x->tensor.shape.size()) - 1) {
    return Status::Unsupported("only last-axis LayerNormalization is supported");
  }
  return Status::OK();
}

Status InferLayerNorm(Graph* graph, const Node& node) {
  if (node.inputs().size() < 2 || node.inputs().size() > 3) {
    return Status::ShapeError("LayerNormalization expects input, scale and optional bias");
  }
  const std::string* bias = node.inputs().size() == 3 ? &node.inputs()[2] : nullptr;
  CUTRITON_RETURN_IF_ERROR(CheckNormParams(*graph, node.inputs()[0], node.inputs()[1], bias,
                                           GetIntAttribute(node, "axis", -1)));
  return graph->SetValueDesc(node.outputs()[0], graph->FindValue(node.inputs()[0])->tensor);
}

Status InferSkipLayerNorm(Graph* graph, const Node& node) {
  if (node.inputs().size() != 4) {
    return Status::ShapeError("SkipLayerNormalization expects input, residual, scale and bias");
  }
  const ValueDesc* x = graph->FindValue(node.inputs()[0]);
  const ValueDesc* r = graph->FindValue(node.inputs()[1]);
  if (x == nullptr || r == nullptr || x->tensor.shape != r->tensor.shape ||
      x->tensor.dtype != r->tensor.dtype || x->tensor.layout != r->tensor.layout) {
    return Status::ShapeError("SkipLayerNormalization input and residual must match");
  }
  CUTRITON_RETURN_IF_ERROR(CheckNormParams(*graph, node.inputs()[0], node.inputs()[2],
                                           &node.inputs()[3], GetIntAttribute(node, "axis", -1)));
  return graph->SetValueDesc(node.outputs()[0], x->tensor);
}

Status InferConvAddRelu(Graph* graph, const Node& node) {
  // inputs: x, w, scale, bias, mean, var, residual
  CUTRITON_RETURN_IF_ERROR(InferConv(graph, node));
  const ValueDesc* out = graph->FindValue(node.outputs()[0]);
  const ValueDesc* residual = graph->FindValue(node.inputs()[6]);
  if (residual == nullptr || residual->tensor.shape != out->tensor.shape ||
      residual->tensor.dtype != out->tensor.dtype) {
    return Status::ShapeError("fused residual must match the convolution output");
  }
  return Status::OK();
}

// ---- passes -----------------------------------------------------------------

class TopologicalSortPass final : public GraphPass {
 public:
  const char* name() const override { return "topological_sort"; }
  Status Run(Graph* graph) const override { return graph->TopologicalSort(); }
};

class ShapeInferencePass final : public GraphPass {
 public:
  const char* name() const override { return "shape_inference"; }
  Status Run(Graph* graph) const override {
    CUTRITON_RETURN_IF_ERROR(RegisterBuiltinOpSchemas());
    for (const auto& node : graph->nodes()) {
      const auto schema = OpSchemaRegistry::Global().Find(node.op_type());
      if (schema == nullptr) return Status::Unsupported("no shape inference for op " + node.op_type());
      if (node.inputs().size() < schema->min_inputs || node.inputs().size() > schema->max_inputs ||
          node.outputs().size() != schema->outputs) {
        return Status::ShapeError("node arity does not match its op schema: " + node.name());
      }
      CUTRITON_RETURN_IF_ERROR(schema->infer(graph, node));
    }
    return Status::OK();
  }
};

// Placeholder kept so the pipeline shape stays stable; constants carry no
// foldable producers in this IR.
class ConstantFoldingPass final : public GraphPass {
 public:
  const char* name() const override { return "constant_folding"; }
  Status Run(Graph*) const override { return Status::OK(); }
};

class DeadNodeEliminationPass final : public GraphPass {
 public:
  const char* name() const override { return "dead_node_elimination"; }
  Status Run(Graph* graph) const override {
    std::unordered_set<std::string> needed(graph->outputs().begin(), graph->outputs().end());
    std::vector<bool> keep(graph->nodes().size(), false);
    for (auto it = graph->nodes().rbegin(); it != graph->nodes().rend(); ++it) {
      const bool live = std::any_of(it->outputs().begin(), it->outputs().end(),
                                    [&](const std::string& v) { return needed.count(v) != 0; });
      if (!live) continue;
      keep[static_cast<std::size_t>(it->id())] = true;
      needed.insert(it->inputs().begin(), it->inputs().end());
    }
    std::vector<int> dead;
    for (const auto& node : graph->nodes()) {
      if (!keep[static_cast<std::size_t>(node.id())]) dead.push_back(node.id());
    }
    return dead.empty() ? Status::OK() : graph->RemoveNodes(dead);
  }
};

// Returns the single consumer of `value`, or -1.
int SoleConsumer(const std::unordered_map<std::string, std::vector<int>>& consumers,
                 const std::string& value) {
  const auto it = consumers.find(value);
  return (it == consumers.end() || it->second.size() != 1) ? -1 : it->second.front();
}

// Runs `try_fuse` on every node until no rewrite happens; each rewrite
// restarts the scan because node ids change.
template <typename Fn>
Status RewriteToFixpoint(Graph* graph, Fn try_fuse) {
  for (bool changed = true; changed;) {
    changed = false;
    const auto consumers = graph->BuildConsumerMap();
    for (auto& node : graph->mutable_nodes()) {
      std::vector<int> removed;
      if (!try_fuse(graph, consumers, node, &removed)) continue;
      CUTRITON_RETURN_IF_ERROR(graph->RemoveNodes(removed));
      changed = true;
      break;
    }
  }
  return Status::OK();
}

class ConvBatchNormReluFusionPass final : public GraphPass {
 public:
  const char* name() const override { return "conv_batchnorm_relu_fusion"; }
  Status Run(Graph* graph) const override {
    return RewriteToFixpoint(graph, [](Graph* g, const auto& consumers, Node& conv,
                                       std::vector<int>* removed) {
      if (conv.op_type() != "Conv" || conv.outputs().size() != 1) return false;
      const int bn_id = SoleConsumer(consumers, conv.outputs()[0]);
      if (bn_id < 0) return false;
      const Node& bn = g->nodes()[static_cast<std::size_t>(bn_id)];
      if (bn.op_type() != "BatchNormalization" || bn.outputs().size() != 1) return false;
      const int relu_id = SoleConsumer(consumers, bn.outputs()[0]);
      const bool with_relu = relu_id >= 0 &&
                             g->nodes()[static_cast<std::size_t>(relu_id)].op_type() == "Relu" &&
                             !g->nodes()[static_cast<std::size_t>(relu_id)].outputs().empty();
      std::vector<std::string> inputs = conv.inputs();
      inputs.insert(inputs.end(), bn.inputs().begin() + 1, bn.inputs().end());
      const std::vector<std::string> outputs =
          with_relu ? g->nodes()[static_cast<std::size_t>(relu_id)].outputs() : bn.outputs();
      const double epsilon = bn.GetAttribute<double>("epsilon").value_or(1e-5);
      conv.set_name(conv.name() + (with_relu ? "_bn_relu" : "_bn"));
      conv.set_op_type(with_relu ? "FusedConvBatchNormRelu" : "FusedConvBatchNorm");
      conv.set_inputs(std::move(inputs));
      conv.set_outputs(outputs);
      conv.SetAttribute("fused_batchnorm_relu", with_relu);
      conv.SetAttribute("batchnorm_epsilon", epsilon);
      removed->push_back(bn_id);
      if (with_relu) removed->push_back(relu_id);
      return true;
    });
  }
};

class AddReluFusionPass final : public GraphPass {
 public:
  const char* name() const override { return "add_relu_fusion"; }
  Status Run(Graph* graph) const override {
    return RewriteToFixpoint(graph, [](Graph* g, const auto& consumers, Node& add,
                                       std::vector<int>* removed) {
      if (add.op_type() != "Add" || add.outputs().size() != 1) return false;
      const int relu_id = SoleConsumer(consumers, add.outputs()[0]);
      if (relu_id < 0) return false;
      const Node& relu = g->nodes()[static_cast<std::size_t>(relu_id)];
      if (relu.op_type() != "Relu" || relu.outputs().size() != 1) return false;
      add.set_name(add.name() + "_relu");
      add.set_op_type("AddRelu");
      add.set_outputs(relu.outputs());
      removed->push_back(relu_id);
      return true;
    });
  }
};

// FusedConvBatchNorm whose only consumer is an AddRelu becomes one op whose
// epilogue adds the residual (the AddRelu's other input) and applies ReLU.
class ConvResidualFusionPass final : public GraphPass {
 public:
  const char* name() const override { return "conv_residual_add_relu_fusion"; }
  Status Run(Graph* graph) const override {
    return RewriteToFixpoint(graph, [](Graph* g, const auto& consumers, Node& conv,
                                       std::vector<int>* removed) {
      if (conv.op_type() != "FusedConvBatchNorm" || conv.outputs().size() != 1 ||
          IsGraphOutput(*g, conv.outputs()[0])) {
        return false;
      }
      const int add_id = SoleConsumer(consumers, conv.outputs()[0]);
      if (add_id < 0) return false;
      const Node& add = g->nodes()[static_cast<std::size_t>(add_id)];
      if (add.op_type() != "AddRelu" || add.inputs().size() != 2 || add.outputs().size() != 1) {
        return false;
      }
      const std::string& residual =
          add.inputs()[0] == conv.outputs()[0] ? add.inputs()[1] : add.inputs()[0];
      if (residual == conv.outputs()[0]) return false;
      // The residual must be produced before the conv runs; the later
      // topological sort enforces it, a self-dependency is rejected here.
      std::vector<std::string> inputs = conv.inputs();
      inputs.push_back(residual);
      conv.set_name(conv.name() + "_add_relu");
      conv.set_op_type("FusedConvBatchNormAddRelu");
      conv.set_inputs(std::move(inputs));
      conv.set_outputs(add.outputs());
      removed->push_back(add_id);
      return true;
    });
  }
};

class GemmGeluFusionPass final : public GraphPass {
 public:
  const char* name() const override { return "gemm_gelu_fusion"; }
  Status Run(Graph* graph) const override {
    return RewriteToFixpoint(graph, [](Graph* g, const auto& consumers, Node& gemm,
                                       std::vector<int>* removed) {
      if (gemm.op_type() != "Gemm" || gemm.outputs().size() != 1 ||
          IsGraphOutput(*g, gemm.outputs()[0])) {
        return false;
      }
      const int gelu_id = SoleConsumer(consumers, gemm.outputs()[0]);
      if (gelu_id < 0) return false;
      const Node& gelu = g->nodes()[static_cast<std::size_t>(gelu_id)];
      if (gelu.op_type() != "Gelu" || gelu.inputs().size() != 1 || gelu.outputs().size() != 1) {
        return false;
      }
      gemm.set_name(gemm.name() + "_gelu");
      gemm.set_op_type("GemmGelu");
      gemm.set_outputs(gelu.outputs());
      removed->push_back(gelu_id);
      return true;
    });
  }
};

class SkipLayerNormFusionPass final : public GraphPass {
 public:
  const char* name() const override { return "skip_layer_norm_fusion"; }
  Status Run(Graph* graph) const override {
    return RewriteToFixpoint(graph, [](Graph* g, const auto& consumers, Node& add,
                                       std::vector<int>* removed) {
      if (add.op_type() != "Add" || add.outputs().size() != 1 ||
          IsGraphOutput(*g, add.outputs()[0])) {
        return false;
      }
      const int norm_id = SoleConsumer(consumers, add.outputs()[0]);
      if (norm_id < 0) return false;
      const Node& norm = g->nodes()[static_cast<std::size_t>(norm_id)];
      if (norm.op_type() != "LayerNormalization" || norm.inputs().size() != 3 ||
          norm.outputs().size() != 1 || norm.inputs()[0] != add.outputs()[0]) {
        return false;
      }
      std::vector<std::string> inputs = add.inputs();
      inputs.push_back(norm.inputs()[1]);
      inputs.push_back(norm.inputs()[2]);
      const int64_t axis = GetIntAttribute(norm, "axis", -1);
      const double epsilon = norm.GetAttribute<double>("epsilon").value_or(1e-5);
      add.set_name(add.name() + "_layer_norm");
      add.set_op_type("SkipLayerNormalization");
      add.set_inputs(std::move(inputs));
      add.set_outputs(norm.outputs());
      add.SetAttribute("axis", axis);
      add.SetAttribute("epsilon", epsilon);
      removed->push_back(norm_id);
      return true;
    });
  }
};

class FlattenGemmNormalizationPass final : public GraphPass {
 public:
  const char* name() const override { return "flatten_gemm_normalization"; }
  Status Run(Graph* graph) const override {
    for (auto& node : graph->mutable_nodes()) {
      if (node.op_type() == "MatMul") {
        node.set_op_type("Gemm");
        node.SetAttribute("normalized_from_matmul", true);
      }
      if (node.op_type() == "Flatten" && !node.GetAttribute<int64_t>("axis")) {
        node.SetAttribute("axis", int64_t{1});
      }
    }
    return Status::OK();
  }
};

class StaticShapeValidationPass final : public GraphPass {
 public:
  const char* name() const override { return "static_shape_validation"; }
  Status Run(Graph* graph) const override {
    for (const auto& entry : graph->values()) {
      const ValueDesc& value = entry.second;
      if (value.tensor.dtype == DataType::kUnknown && !value.is_constant) continue;
      if (!value.tensor.shape.empty()) CUTRITON_RETURN_IF_ERROR(value.tensor.Validate());
    }
    for (const auto& output : graph->outputs()) {
      const ValueDesc* value = graph->FindValue(output);
      if (value == nullptr) return Status::NotFound("graph output is missing: " + output);
      CUTRITON_RETURN_IF_ERROR(value->tensor.Validate());
    }
    return Status::OK();
  }
};

}  // namespace

Status RegisterBuiltinOpSchemas() {
  auto& registry = OpSchemaRegistry::Global();
  auto add = [&](const char* op, std::size_t lo, std::size_t hi, ShapeInferenceFunction fn) {
    const Status status = registry.Register(OpSchema{op, lo, hi, 1, std::move(fn)});
    return status.code() == ErrorCode::kAlreadyExists ? Status::OK() : status;
  };
  CUTRITON_RETURN_IF_ERROR(add("Conv", 2, 2, InferConv));
  CUTRITON_RETURN_IF_ERROR(add("FusedConvBatchNorm", 6, 6, InferConv));
  CUTRITON_RETURN_IF_ERROR(add("FusedConvBatchNormRelu", 6, 6, InferConv));
  CUTRITON_RETURN_IF_ERROR(add("FusedConvBatchNormAddRelu", 7, 7, InferConvAddRelu));
  CUTRITON_RETURN_IF_ERROR(add("BatchNormalization", 5, 5, InferLikeFirstInput));
  for (const char* op : {"Relu", "Gelu", "Softmax"}) {
    CUTRITON_RETURN_IF_ERROR(add(op, 1, 1, InferLikeFirstInput));
  }
  CUTRITON_RETURN_IF_ERROR(add("LayerNormalization", 2, 3, InferLayerNorm));
  CUTRITON_RETURN_IF_ERROR(add("Add", 2, 2, InferBinary));
  CUTRITON_RETURN_IF_ERROR(add("AddRelu", 2, 2, InferBinary));
  CUTRITON_RETURN_IF_ERROR(add("Flatten", 1, 1, InferFlatten));
  CUTRITON_RETURN_IF_ERROR(add("Gemm", 2, 3, InferGemm));
  CUTRITON_RETURN_IF_ERROR(add("GemmGelu", 2, 3, InferGemm));
  CUTRITON_RETURN_IF_ERROR(add("MatMul", 2, 2, InferGemm));
  CUTRITON_RETURN_IF_ERROR(add("SkipLayerNormalization", 4, 4, InferSkipLayerNorm));
  CUTRITON_RETURN_IF_ERROR(add("MaxPool", 1, 1, InferPool));
  CUTRITON_RETURN_IF_ERROR(add("AveragePool", 1, 1, InferPool));
  CUTRITON_RETURN_IF_ERROR(add("GlobalAveragePool", 1, 1, InferGlobalAveragePool));
  CUTRITON_RETURN_IF_ERROR(add("Constant", 0, 0, [](Graph*, const Node&) { return Status::OK(); }));
  // Diagnostic op of this backend: y = x after a bounded wait that always
  // expires (exercises the kernel error block; see kernels/diag.cu).
  CUTRITON_RETURN_IF_ERROR(add("BoundedWaitProbe", 1, 1, InferLikeFirstInput));
  return Status::OK();
}

void PassManager::Add(std::unique_ptr<GraphPass> pass) { passes_.push_back(std::move(pass)); }

Status PassManager::Run(Graph* graph) const {
  executed_passes_.clear();
  for (const auto& pass : passes_) {
    CUTRITON_RETURN_IF_ERROR(pass->Run(graph));
    executed_passes_.push_back(pass->name());
  }
  return Status::OK();
}

std::unique_ptr<GraphPass> CreateTopologicalSortPass() { return std::make_unique<TopologicalSortPass>(); }
std::unique_ptr<GraphPass> CreateShapeInferencePass() { return std::make_unique<ShapeInferencePass>(); }
std::unique_ptr<GraphPass> CreateConstantFoldingPass() { return std::make_unique<ConstantFoldingPass>(); }
std::unique_ptr<GraphPass> CreateDeadNodeEliminationPass() { return std::make_unique<DeadNodeEliminationPass>(); }
std::unique_ptr<GraphPass> CreateConvBatchNormReluFusionPass() { return std::make_unique<ConvBatchNormReluFusionPass>(); }
std::unique_ptr<GraphPass> CreateAddReluFusionPass() { return std::make_unique<AddReluFusionPass>(); }
std::unique_ptr<GraphPass> CreateGemmGeluFusionPass() { return std::make_unique<GemmGeluFusionPass>(); }
std::unique_ptr<GraphPass> CreateSkipLayerNormalizationFusionPass() { return std::make_unique<SkipLayerNormFusionPass>(); }
std::unique_ptr<GraphPass> CreateFlattenGemmNormalizationPass() { return std::make_unique<FlattenGemmNormalizationPass>(); }
std::unique_ptr<GraphPass> CreateStaticShapeValidationPass() { return std::make_unique<StaticShapeValidationPass>(); }
std::unique_ptr<GraphPass> CreateConvResidualFusionPass() { return std::make_unique<ConvResidualFusionPass>(); }

PassManager CreateDefaultCompilePasses(bool enable_transformer_fusions) {
  return CreateCompilePasses(enable_transformer_fusions, false);
}

PassManager CreateCompilePasses(bool enable_transformer_fusions, bool enable_residual_fusion) {
  PassManager manager;
  manager.Add(CreateTopologicalSortPass());
  manager.Add(CreateShapeInferencePass());
  manager.Add(CreateConstantFoldingPass());
  manager.Add(CreateDeadNodeEliminationPass());
  manager.Add(CreateConvBatchNormReluFusionPass());
  manager.Add(CreateAddReluFusionPass());
  if (enable_residual_fusion) manager.Add(CreateConvResidualFusionPass());
  if (enable_transformer_fusions) {
    manager.Add(CreateGemmGeluFusionPass());
    manager.Add(CreateSkipLayerNormalizationFusionPass());
  }
  manager.Add(CreateTopologicalSortPass());
  manager.Add(CreateShapeInferencePass());
  manager.Add(CreateFlattenGemmNormalizationPass());
  manager.Add(CreateDeadNodeEliminationPass());
  manager.Add(CreateStaticShapeValidationPass());
  return manager;
}

}  // namespace cutriton
