// Backend registry, the cpu_reference stub and the cuda_sm100 lowering.
//
// Lowering follows the reference's CudaTritonBackend::Lower
// (src/backend/backend.cpp:235-362): every pack variant that matches the
// node's dtype/layout/SM and constraints becomes one candidate, and each
// FusionRegistry decomposition of a fused op becomes one more candidate built
// from the sub-ops' kernels, with scratch temporaries in shared slots. The
// sub-op kernel is the sub-op's default variant when its constraints hold,
// else the first variant whose constraints hold (the reference always takes
// the default; packs here carry shape-specialised tcgen05 variants).

#include "cutriton/backend/backend.h"

#include <algorithm>
#include <cstdlib>
#include <functional>
#include <mutex>

#include "../cuda_driver.h"
#include "cutriton/ir/fusion.h"
#include "cutriton/ir/op_schema.h"

namespace cutriton {
namespace {

constexpr const char* kCudaBackendName = "cuda_sm100";

using ValueLookup = std::function<const ValueDesc*(const std::string&)>;

class UnsupportedCpuBackend final : public Backend {
 public:
  const char* name() const override { return "cpu_reference"; }
  Status CheckSupport(const Node&, const Graph&, const BackendOptions&) const override {
    return Status::Unsupported("the CPU reference backend has no production kernels");
  }
  Status CreateKernel(const Node&, const Graph&, const BackendOptions&,
                      std::unique_ptr<OpKernel>*) const override {
    return Status::Unsupported("the CPU reference backend has no production kernels");
  }
};

// Flatten: the memory planner aliases output to input; nothing to launch.
class ViewKernel final : public OpKernel {
 public:
  const char* backend_name() const override { return kCudaBackendName; }
  const char* op_type() const override { return "Flatten"; }
  Status Compute(KernelContext* context) override {
    if (context == nullptr || context->node == nullptr || context->tensors == nullptr) {
      return Status::InvalidArgument("Flatten kernel context is invalid");
    }
    return Status::OK();
  }
};

// Compute capability of the target device. Without a driver (build hosts)
// the environment variable CUTRITON_ASSUME_COMPUTE_CAPABILITY lets lowering
// run for plan-inspection tests; execution still needs the device.
Status TargetCapability(int device_id, int* capability) {
  Status status = drv::ComputeCapability(device_id, capability);
  if (status.ok()) return status;
  if (const char* assumed = std::getenv("CUTRITON_ASSUME_COMPUTE_CAPABILITY")) {
    *capability = std::atoi(assumed);
    if (*capability > 0) return Status::OK();
  }
  return status;
}

Status CheckTensor(const Graph& graph, const std::string& name, const Device& device) {
  const ValueDesc* value = graph.FindValue(name);
  if (value == nullptr) return Status::NotFound("tensor description is missing: " + name);
  CUTRITON_RETURN_IF_ERROR(value->tensor.Validate());
  if (value->tensor.dtype != DataType::kFloat32 && value->tensor.dtype != DataType::kFloat16) {
    return Status::Unsupported("only float32/float16 tensors are supported: " + name);
  }
  if (value->tensor.device_type != device.type || value->tensor.device_id != device.id) {
    return Status::Unsupported("tensor is assigned to another device: " + name);
  }
  return Status::OK();
}

bool ConstraintHolds(const KernelConstraint& c, const Node& node, const ValueLookup& lookup) {
  switch (c.kind) {
    case KernelConstraintKind::kInputCountEquals:
      return node.inputs().size() == static_cast<std::size_t>(c.expected);
    case KernelConstraintKind::kAttributeInt64Equals:
      return GetIntAttribute(node, c.attribute_name, c.default_value) == c.expected;
    case KernelConstraintKind::kAttributeListEquals:
      return GetIntListAttribute(node, c.attribute_name, c.default_list) == c.expected_list;
    case KernelConstraintKind::kInputIsConstant: {
      if (c.tensor_index < 0 || static_cast<std::size_t>(c.tensor_index) >= node.inputs().size()) return false;
      const ValueDesc* v = lookup(node.inputs()[static_cast<std::size_t>(c.tensor_index)]);
      return v != nullptr && v->is_constant;
    }
    case KernelConstraintKind::kTensorRankEquals:
    case KernelConstraintKind::kDimMultipleOf:
    case KernelConstraintKind::kDimLessEqual: {
      const auto& names = c.tensor_is_output ? node.outputs() : node.inputs();
      if (c.tensor_index < 0 || static_cast<std::size_t>(c.tensor_index) >= names.size()) return false;
      const ValueDesc* v = lookup(names[static_cast<std::size_t>(c.tensor_index)]);
      if (v == nullptr) return false;
      const auto& shape = v->tensor.shape;
      if (c.kind == KernelConstraintKind::kTensorRankEquals) {
        return shape.size() == static_cast<std::size_t>(c.expected);
      }
      if (c.axis < 0 || static_cast<std::size_t>(c.axis) >= shape.size()) return false;
      const int64_t dim = shape[static_cast<std::size_t>(c.axis)];
      return c.kind == KernelConstraintKind::kDimMultipleOf ? dim % c.expected == 0
                                                           : dim <= c.expected;
    }
  }
  return false;
}

bool ArtifactMatches(const KernelArtifact& artifact, const Node& node, const ValueLookup& lookup,
                     int capability) {
  if (capability < artifact.min_compute_capability) return false;
  const std::string& reference_name = node.outputs().empty() ? node.inputs().front() : node.outputs().front();
  const ValueDesc* reference = lookup(reference_name);
  if (reference == nullptr || artifact.dtype != DataTypeName(reference->tensor.dtype)) return false;
  auto layout_ok = [&](const std::string& name) {
    const ValueDesc* v = lookup(name);
    return v != nullptr && (artifact.layout.empty() || v->tensor.layout == artifact.layout);
  };
  if (!node.inputs().empty() && !layout_ok(node.inputs().front())) return false;
  for (const auto& output : node.outputs()) {
    if (!layout_ok(output)) return false;
  }
  // A prepacked argument can only bind a constant input.
  for (const auto& arg : artifact.arguments) {
    if (arg.source.prepack.empty()) continue;
    if (arg.source.index < 0 || static_cast<std::size_t>(arg.source.index) >= node.inputs().size()) return false;
    const ValueDesc* v = lookup(node.inputs()[static_cast<std::size_t>(arg.source.index)]);
    if (v == nullptr || !v->is_constant) return false;
  }
  return std::all_of(artifact.constraints.begin(), artifact.constraints.end(),
                     [&](const KernelConstraint& c) { return ConstraintHolds(c, node, lookup); });
}

Status CheckCudaNode(const Node& node, const Graph& graph, const BackendOptions& options,
                     const ArtifactRepository& repository, int* capability) {
  if (options.device.type != DeviceType::kCUDA) {
    return Status::Unsupported("cuda_sm100 requires a CUDA device");
  }
  CUTRITON_RETURN_IF_ERROR(RegisterBuiltinOpSchemas());
  const auto schema = OpSchemaRegistry::Global().Find(node.op_type());
  if (schema == nullptr) return Status::Unsupported("no op schema is registered for " + node.op_type());
  if (node.inputs().size() < schema->min_inputs || node.inputs().size() > schema->max_inputs ||
      node.outputs().size() != schema->outputs) {
    return Status::Unsupported(node.op_type() + " has an invalid input/output count");
  }
  for (const auto& name : node.inputs()) CUTRITON_RETURN_IF_ERROR(CheckTensor(graph, name, options.device));
  for (const auto& name : node.outputs()) CUTRITON_RETURN_IF_ERROR(CheckTensor(graph, name, options.device));
  if (node.op_type() == "Flatten") {
    const auto& outs = graph.outputs();
    if (std::find(outs.begin(), outs.end(), node.outputs().front()) != outs.end()) {
      return Status::Unsupported("a Flatten graph output would need an explicit copy kernel");
    }
    return Status::OK();
  }
  const auto* artifacts = repository.Find(node.op_type());
  if (artifacts == nullptr || artifacts->empty()) {
    // A fused op without its own kernel may still lower through its
    // decomposition; Lower decides.
    if (FusionRegistry::Global().Find(node.op_type()).empty()) {
      return Status::Unsupported("no Kernel Pack entry for " + node.op_type());
    }
  }
  CUTRITON_RETURN_IF_ERROR(TargetCapability(options.device.id, capability));
  if (artifacts == nullptr) return Status::OK();
  const ValueLookup lookup = [&](const std::string& n) { return graph.FindValue(n); };
  for (const auto& artifact : *artifacts) {
    if (ArtifactMatches(artifact, node, lookup, *capability)) return Status::OK();
  }
  if (!FusionRegistry::Global().Find(node.op_type()).empty()) return Status::OK();
  return Status::Unsupported("no Kernel Pack variant of " + node.op_type() +
                             " matches dtype/layout/SM/constraints");
}

// Kernel for one step of an unfused decomposition: the default variant if its
// constraints hold for the synthesized sub-node, else another variant of the
// default kernel, else the first that matches.
const KernelArtifact* PickSubKernel(const ArtifactRepository& repository, const Node& sub,
                                    const std::string& dtype, const ValueLookup& lookup,
                                    int capability) {
  const auto* list = repository.Find(sub.op_type());
  if (list == nullptr) return nullptr;
  std::string default_kernel;
  for (const auto& a : *list) {
    if (a.dtype == dtype && a.is_default) default_kernel = a.kernel_id;
  }
  const KernelArtifact* sibling = nullptr;
  const KernelArtifact* fallback = nullptr;
  for (const auto& a : *list) {
    if (a.dtype != dtype || !ArtifactMatches(a, sub, lookup, capability)) continue;
    if (a.is_default) return &a;
    if (sibling == nullptr && a.kernel_id == default_kernel) sibling = &a;
    if (fallback == nullptr) fallback = &a;
  }
  return sibling != nullptr ? sibling : fallback;
}

class CudaSm100Backend final : public Backend {
 public:
  const char* name() const override { return kCudaBackendName; }

  Status CheckSupport(const Node& node, const Graph& graph,
                      const BackendOptions& options) const override {
    ArtifactRepository repository;
    std::vector<std::string> paths = options.kernel_artifact_paths;
    if (paths.empty() && !options.kernel_artifact_dir.empty()) paths.push_back(options.kernel_artifact_dir);
    CUTRITON_RETURN_IF_ERROR(repository.Load(paths));
    int capability = 0;
    return CheckCudaNode(node, graph, options, repository, &capability);
  }

  Status Lower(const Node& node, const LoweringContext& context,
               std::vector<ExecutionCandidate>* candidates) const override {
    if (candidates == nullptr || context.graph == nullptr || context.options == nullptr ||
        context.artifacts == nullptr || context.catalog == nullptr) {
      return Status::InvalidArgument("CUDA lowering context is incomplete");
    }
    const Graph& graph = *context.graph;
    int capability = 0;
    CUTRITON_RETURN_IF_ERROR(CheckCudaNode(node, graph, *context.options, *context.artifacts, &capability));
    candidates->clear();
    if (node.op_type() == "Flatten") {
      ExecutionCandidate view;
      view.candidate_id = "view:flatten";
      view.is_default = true;
      view.steps.push_back(ViewInvocation{node.inputs().front(), node.outputs().front()});
      candidates->push_back(std::move(view));
      return Status::OK();
    }
    const ValueDesc* out = graph.FindValue(node.outputs().front());
    if (out == nullptr) return Status::NotFound("lowered node output description is missing");
    const std::string dtype = DataTypeName(out->tensor.dtype);
    const std::string layout = node.inputs().empty() ? std::string{}
                                                     : graph.FindValue(node.inputs().front())->tensor.layout;
    const ValueLookup lookup = [&](const std::string& n) { return graph.FindValue(n); };
    const auto artifacts = context.catalog->Query(node.op_type(), dtype, layout, capability);
    std::string default_kernel;  // kernel_id of the op's default variant, matching or not
    for (const KernelArtifact* artifact : artifacts) {
      if (artifact->is_default) default_kernel = artifact->kernel_id;
    }
    std::vector<std::string> kernel_ids;
    for (const KernelArtifact* artifact : artifacts) {
      if (!ArtifactMatches(*artifact, node, lookup, capability)) continue;
      ExecutionCandidate candidate;
      candidate.candidate_id = artifact->identity();
      candidate.is_default = artifact->is_default;
      candidate.steps.push_back(KernelInvocation{*artifact, node.inputs(), node.outputs()});
      candidates->push_back(std::move(candidate));
      kernel_ids.push_back(artifact->kernel_id);
    }
    // Without a matching default variant, another variant of the default
    // kernel leads (a shape-specialised default falls back to its general
    // sibling); failing that, the first matching candidate.
    if (!candidates->empty() &&
        std::none_of(candidates->begin(), candidates->end(),
                     [](const ExecutionCandidate& c) { return c.is_default; })) {
      std::size_t lead = 0;
      for (std::size_t i = 0; i < kernel_ids.size(); ++i) {
        if (!default_kernel.empty() && kernel_ids[i] == default_kernel) {
          lead = i;
          break;
        }
      }
      (*candidates)[lead].is_default = true;
    }
    CUTRITON_RETURN_IF_ERROR(RegisterBuiltinFusionAlternatives());
    for (const auto& alternative : FusionRegistry::Global().Find(node.op_type())) {
      ExecutionCandidate candidate;
      if (BuildDecomposition(node, alternative, graph, *context.artifacts, dtype, capability, &candidate)) {
        if (candidates->empty()) candidate.is_default = true;
        candidates->push_back(std::move(candidate));
      }
    }
    return candidates->empty() ? Status::Unsupported("no compatible artifact for " + node.op_type())
                               : Status::OK();
  }

  Status CreateKernel(const Node& node, const Graph&, const BackendOptions&,
                      std::unique_ptr<OpKernel>* kernel) const override {
    if (kernel == nullptr) return Status::InvalidArgument("OpKernel output pointer is null");
    if (node.op_type() == "Flatten") {
      *kernel = std::make_unique<ViewKernel>();
      return Status::OK();
    }
    return Status::Unsupported("artifact-backed kernels are created from KernelInvocation");
  }

 private:
  // One step of a decomposition: a sub-op node plus the kernel chosen for it.
  struct Step {
    std::string op_type;
    std::vector<std::string> inputs;
    std::vector<std::string> outputs;
  };

  static bool BuildDecomposition(const Node& node, const FusionAlternative& alternative,
                                 const Graph& graph, const ArtifactRepository& repository,
                                 const std::string& dtype, int capability,
                                 ExecutionCandidate* candidate) {
    const std::string& op = node.op_type();
    const auto& in = node.inputs();
    const std::string& out = node.outputs().front();
    std::vector<Step> steps;
    std::vector<CandidateTemporary> temporaries;
    auto temp = [&](const char* suffix, std::size_t slot) {
      const std::string name = node.name() + "::__" + suffix;
      temporaries.push_back(CandidateTemporary{name, out, slot});
      return name;
    };
    if (op == "FusedConvBatchNormRelu" || op == "FusedConvBatchNorm") {
      const std::string conv = temp("conv", 0);
      steps.push_back({"Conv", {in[0], in[1]}, {conv}});
      if (op == "FusedConvBatchNormRelu") {
        const std::string bn = temp("bn", 1);
        steps.push_back({"BatchNormalization", {conv, in[2], in[3], in[4], in[5]}, {bn}});
        steps.push_back({"Relu", {bn}, {out}});
      } else {
        steps.push_back({"BatchNormalization", {conv, in[2], in[3], in[4], in[5]}, {out}});
      }
    } else if (op == "FusedConvBatchNormAddRelu") {
      const std::string conv_bn = temp("conv_bn", 0);
      steps.push_back({"FusedConvBatchNorm", {in[0], in[1], in[2], in[3], in[4], in[5]}, {conv_bn}});
      steps.push_back({"AddRelu", {conv_bn, in[6]}, {out}});
    } else if (op == "AddRelu") {
      const std::string sum = temp("add", 0);
      steps.push_back({"Add", in, {sum}});
      steps.push_back({"Relu", {sum}, {out}});
    } else if (op == "GemmGelu") {
      const std::string projected = temp("gemm", 0);
      steps.push_back({"Gemm", in, {projected}});
      steps.push_back({"Gelu", {projected}, {out}});
    } else if (op == "SkipLayerNormalization") {
      const std::string sum = temp("add", 0);
      steps.push_back({"Add", {in[0], in[1]}, {sum}});
      steps.push_back({"LayerNormalization", {sum, in[2], in[3]}, {out}});
    } else {
      return false;
    }
    // Temporaries look like the fused output for constraint checks.
    const ValueLookup lookup = [&](const std::string& n) -> const ValueDesc* {
      for (const auto& t : temporaries) {
        if (t.name == n) return graph.FindValue(t.like_value);
      }
      return graph.FindValue(n);
    };
    candidate->candidate_id = alternative.candidate_id;
    candidate->temporaries = temporaries;
    for (const auto& step : steps) {
      Node sub(node.name() + "::" + step.op_type, step.op_type, step.inputs, step.outputs);
      for (const auto& attr : node.attributes()) sub.SetAttribute(attr.first, attr.second);
      if (const auto eps = node.GetAttribute<double>("batchnorm_epsilon")) sub.SetAttribute("epsilon", *eps);
      const KernelArtifact* artifact = PickSubKernel(repository, sub, dtype, lookup, capability);
      if (artifact == nullptr) return false;
      candidate->steps.push_back(KernelInvocation{*artifact, step.inputs, step.outputs});
    }
    return true;
  }
};

Status RegisterIfMissing(std::shared_ptr<Backend> backend) {
  auto& registry = KernelRegistry::Global();
  if (registry.GetBackend(backend->name()) != nullptr) return Status::OK();
  const Status status = registry.RegisterBackend(std::move(backend));
  return status.code() == ErrorCode::kAlreadyExists ? Status::OK() : status;
}

}  // namespace

Status Backend::Lower(const Node& node, const LoweringContext& context,
                      std::vector<ExecutionCandidate>* candidates) const {
  if (candidates == nullptr || context.graph == nullptr || context.options == nullptr) {
    return Status::InvalidArgument("lowering context is incomplete");
  }
  CUTRITON_RETURN_IF_ERROR(CheckSupport(node, *context.graph, *context.options));
  ExecutionCandidate candidate;
  candidate.candidate_id = std::string(name()) + ":legacy:" + node.op_type();
  candidate.is_default = true;
  candidates->assign(1, std::move(candidate));
  return Status::OK();
}

KernelRegistry& KernelRegistry::Global() {
  static KernelRegistry registry;
  return registry;
}

Status KernelRegistry::RegisterBackend(std::shared_ptr<Backend> backend) {
  if (backend == nullptr) return Status::InvalidArgument("backend must not be null");
  const std::string name = backend->name();
  if (name.empty()) return Status::InvalidArgument("backend name must not be empty");
  std::unique_lock<std::shared_mutex> lock(mutex_);
  if (!backends_.emplace(name, std::move(backend)).second) {
    return Status::AlreadyExists("backend is already registered: " + name);
  }
  return Status::OK();
}

std::shared_ptr<Backend> KernelRegistry::GetBackend(const std::string& name) const {
  std::shared_lock<std::shared_mutex> lock(mutex_);
  const auto it = backends_.find(name);
  return it == backends_.end() ? nullptr : it->second;
}

std::vector<std::string> KernelRegistry::AvailableBackends() const {
  std::shared_lock<std::shared_mutex> lock(mutex_);
  std::vector<std::string> names;
  for (const auto& entry : backends_) names.push_back(entry.first);
  std::sort(names.begin(), names.end());
  return names;
}

void KernelRegistry::ClearForTests() {
  std::unique_lock<std::shared_mutex> lock(mutex_);
  backends_.clear();
}

std::shared_ptr<Backend> CreateCpuReferenceBackend() { return std::make_shared<UnsupportedCpuBackend>(); }
std::shared_ptr<Backend> CreateCudaSm100Backend() { return std::make_shared<CudaSm100Backend>(); }
std::shared_ptr<Backend> CreateCudaTritonBackend() { return CreateCudaSm100Backend(); }

Status RegisterBuiltinBackends() {
  CUTRITON_RETURN_IF_ERROR(RegisterIfMissing(CreateCpuReferenceBackend()));
  CUTRITON_RETURN_IF_ERROR(RegisterIfMissing(CreateCudaSm100Backend()));
  return Status::OK();
}

bool IsCudaArtifactTarget(const std::string& target) {
  return target == kCudaBackendName || target == "cuda_triton";
}

std::string CanonicalTargetName(const std::string& target) {
  return target == "cuda_triton" ? std::string(kCudaBackendName) : target;
}

}  // namespace cutriton
