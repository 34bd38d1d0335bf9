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

// Why the value `name` cannot take part in a cuda_sm100 launch, or "".
std::string TensorProblem(const Graph& graph, const std::string& name, const Device& device) {
  const ValueDesc* value = graph.FindValue(name);
  if (value == nullptr) return "'" + name + "' has no description";
  const Status valid = value->tensor.Validate();
  if (!valid.ok()) return "'" + name + "': " + valid.message();
  const DataType dtype = value->tensor.dtype;
  if (dtype != DataType::kFloat32 && dtype != DataType::kFloat16) {
    return "'" + name + "' is " + DataTypeName(dtype) + " (kernels take float32 / float16)";
  }
  if (value->tensor.device_type != device.type || value->tensor.device_id != device.id) {
    return "'" + name + "' is placed on another device";
  }
  return "";
}

bool ConstraintHolds(const KernelConstraint& c, const Node& node, const ValueLookup& lookup) {
  const auto pick = [&](bool output) -> const ValueDesc* {
    const auto& names = output ? node.outputs() : node.inputs();
    if (c.tensor_index < 0 || static_cast<std::size_t>(c.tensor_index) >= names.size()) return nullptr;
    return lookup(names[static_cast<std::size_t>(c.tensor_index)]);
  };
  switch (c.kind) {
    case KernelConstraintKind::kInputCountEquals:
      return static_cast<int64_t>(node.inputs().size()) == c.expected;
    case KernelConstraintKind::kAttributeInt64Equals:
      return GetIntAttribute(node, c.attribute_name, c.default_value) == c.expected;
    case KernelConstraintKind::kAttributeListEquals:
      return GetIntListAttribute(node, c.attribute_name, c.default_list) == c.expected_list;
    case KernelConstraintKind::kInputIsConstant: {
      const ValueDesc* v = pick(false);
      return v != nullptr && v->is_constant;
    }
    case KernelConstraintKind::kTensorRankEquals: {
      const ValueDesc* v = pick(c.tensor_is_output);
      return v != nullptr && static_cast<int64_t>(v->tensor.shape.size()) == c.expected;
    }
    case KernelConstraintKind::kDimMultipleOf:
    case KernelConstraintKind::kDimLessEqual: {
      const ValueDesc* v = pick(c.tensor_is_output);
      if (v == nullptr || c.axis < 0 || static_cast<std::size_t>(c.axis) >= v->tensor.shape.size()) return false;
      const int64_t dim = v->tensor.shape[static_cast<std::size_t>(c.axis)];
      return c.kind == KernelConstraintKind::kDimMultipleOf ? dim % c.expected == 0 : dim <= c.expected;
    }
  }
  return false;
}

// Why pack variant `artifact` cannot run `node` on a device of compute
// capability `capability`, or "" when it can. Checked in order: SM, the
// element type of the node's first output (first input for output-less
// nodes), the layout of the first input and of every output, prepacked
// arguments binding constants, then every constraint of the entry.
std::string VariantProblem(const KernelArtifact& artifact, const Node& node, const ValueLookup& lookup,
                           int capability) {
  if (capability < artifact.min_compute_capability) {
    return "needs sm_" + std::to_string(artifact.min_compute_capability);
  }
  const std::string& typed = node.outputs().empty() ? node.inputs().front() : node.outputs().front();
  const ValueDesc* typed_value = lookup(typed);
  if (typed_value == nullptr) return "'" + typed + "' has no description";
  if (artifact.dtype != DataTypeName(typed_value->tensor.dtype)) return "is a " + artifact.dtype + " kernel";
  std::vector<std::string> laid_out(node.outputs().begin(), node.outputs().end());
  if (!node.inputs().empty()) laid_out.push_back(node.inputs().front());
  for (const std::string& name : laid_out) {
    const ValueDesc* v = lookup(name);
    if (v == nullptr) return "'" + name + "' has no description";
    if (!artifact.layout.empty() && v->tensor.layout != artifact.layout) {
      return "wants layout " + artifact.layout + " for '" + name + "'";
    }
  }
  for (const auto& argument : artifact.arguments) {
    if (argument.source.prepack.empty()) continue;
    const int slot = argument.source.index;
    const ValueDesc* v =
        slot >= 0 && static_cast<std::size_t>(slot) < node.inputs().size() ? lookup(node.inputs()[slot]) : nullptr;
    if (v == nullptr || !v->is_constant) return "prepacks argument '" + argument.name + "', which is not a constant";
  }
  for (std::size_t i = 0; i < artifact.constraints.size(); ++i) {
    if (!ConstraintHolds(artifact.constraints[i], node, lookup)) return "constraint " + std::to_string(i) + " fails";
  }
  return "";
}

bool ArtifactMatches(const KernelArtifact& artifact, const Node& node, const ValueLookup& lookup, int capability) {
  return VariantProblem(artifact, node, lookup, capability).empty();
}

// Node-level admission for cuda_sm100: a CUDA device, a schema whose arity
// the node meets, float tensors on the plan's device, and either a pack
// variant that can run it or (fused ops) a registered decomposition.
// `capability` receives the target's compute capability.
Status CheckCudaNode(const Node& node, const Graph& graph, const BackendOptions& options,
                     const ArtifactRepository& repository, int* capability) {
  const std::string who = "cuda_sm100, node '" + node.name() + "' (" + node.op_type() + "): ";
  if (options.device.type != DeviceType::kCUDA) return Status::Unsupported(who + "the plan is not on a CUDA device");
  CUTRITON_RETURN_IF_ERROR(RegisterBuiltinOpSchemas());
  const auto schema = OpSchemaRegistry::Global().Find(node.op_type());
  if (schema == nullptr) return Status::Unsupported(who + "unknown op type");
  const std::size_t ins = node.inputs().size();
  if (ins < schema->min_inputs || ins > schema->max_inputs || node.outputs().size() != schema->outputs) {
    return Status::Unsupported(who + "wrong number of inputs or outputs");
  }
  for (const auto* names : {&node.inputs(), &node.outputs()}) {
    for (const std::string& name : *names) {
      const std::string problem = TensorProblem(graph, name, options.device);
      if (!problem.empty()) return Status::Unsupported(who + problem);
    }
  }
  if (node.op_type() == "Flatten") {
    const auto& outputs = graph.outputs();
    if (std::find(outputs.begin(), outputs.end(), node.outputs().front()) != outputs.end()) {
      return Status::Unsupported(who + "a Flatten that is a graph output would need a copy kernel");
    }
    return Status::OK();
  }
  const bool decomposable = !FusionRegistry::Global().Find(node.op_type()).empty();
  const auto* variants = repository.Find(node.op_type());
  if ((variants == nullptr || variants->empty()) && !decomposable) {
    return Status::Unsupported(who + "the kernel pack has no entry for this op");
  }
  CUTRITON_RETURN_IF_ERROR(TargetCapability(options.device.id, capability));
  if (variants == nullptr || decomposable) return Status::OK();
  const ValueLookup lookup = [&](const std::string& n) { return graph.FindValue(n); };
  std::string reasons;
  for (const KernelArtifact& variant : *variants) {
    const std::string problem = VariantProblem(variant, node, lookup, *capability);
    if (problem.empty()) return Status::OK();
    reasons += (reasons.empty() ? "" : "; ") + variant.identity() + " " + problem;
  }
  return Status::Unsupported(who + "no pack variant fits: " + reasons);
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
