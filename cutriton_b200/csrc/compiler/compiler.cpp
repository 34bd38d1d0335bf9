// Model -> ExecutablePlan.
//
// Same stages as the reference compiler (src/compiler/compiler.cpp:124-284):
// profile validation, passes, device retagging of every typed value for CUDA
// targets, pack loading, lowering of every node into candidates (the default
// candidate selected), then memory planning: static, or per shape profile at
// the profile's max point, plus shared slots for candidate temporaries.
// CUDA-ness is keyed on the backend ("cuda_sm100", alias "cuda_triton"), not on
// a hard-coded target string.

#include "cutriton/compiler/compiler.h"

#include <algorithm>

#include "cutriton/backend/backend.h"
#include "cutriton/ir/pass.h"
#include "cutriton/runtime/memory_planner.h"

namespace cutriton {
namespace {

enum class Point { kMin, kOpt, kMax };

const std::vector<int64_t>& PointOf(const ShapeRange& range, Point p) {
  return p == Point::kMin ? range.min : p == Point::kMax ? range.max : range.opt;
}

Status ValidateProfiles(const Graph& graph, const std::vector<ShapeProfile>& profiles) {
  for (const auto& profile : profiles) {
    if (profile.name.empty()) return Status::InvalidArgument("ShapeProfile name must not be empty");
    for (const auto& input : graph.inputs()) {
      const auto it = profile.inputs.find(input);
      if (it == profile.inputs.end()) return Status::InvalidArgument("ShapeProfile is missing input: " + input);
      const ShapeRange& r = it->second;
      if (r.min.empty() || r.min.size() != r.opt.size() || r.min.size() != r.max.size()) {
        return Status::ShapeError("ShapeProfile ranks differ for " + input);
      }
      for (std::size_t a = 0; a < r.min.size(); ++a) {
        if (r.min[a] <= 0 || r.min[a] > r.opt[a] || r.opt[a] > r.max[a]) {
          return Status::ShapeError("ShapeProfile min/opt/max is invalid for " + input);
        }
      }
    }
  }
  return Status::OK();
}

Status ApplyPoint(Graph* graph, const ShapeProfile& profile, Point point) {
  for (const auto& input : graph->inputs()) {
    const ValueDesc* value = graph->FindValue(input);
    if (value == nullptr) return Status::NotFound("graph input is missing: " + input);
    TensorDesc desc = value->tensor;
    desc.shape = PointOf(profile.inputs.at(input), point);
    CUTRITON_RETURN_IF_ERROR(graph->SetValueDesc(input, std::move(desc)));
  }
  return Status::OK();
}

Status ResolveAt(const Graph& optimized, const ShapeProfile& profile, Point point, Graph* out) {
  *out = optimized;
  CUTRITON_RETURN_IF_ERROR(ApplyPoint(out, profile, point));
  return CreateShapeInferencePass()->Run(out);
}

std::size_t Align256(std::size_t bytes) { return (bytes + 255) / 256 * 256; }

// Candidate temporaries share numbered slots appended after the planned
// workspace; each slot is as large as its largest user.
Status AddCandidateTemporaries(const Graph& graph, const std::vector<PlanOp>& ops, MemoryPlan* plan) {
  std::vector<std::size_t> slot_bytes;
  for (const auto& op : ops) {
    for (const auto& c : op.candidates) {
      for (const auto& t : c.temporaries) {
        const ValueDesc* like = graph.FindValue(t.like_value);
        if (like == nullptr || like->tensor.ByteSize() == 0) {
          return Status::ShapeError("candidate temporary has no concrete shape: " + t.name);
        }
        if (slot_bytes.size() <= t.slot) slot_bytes.resize(t.slot + 1, 0);
        slot_bytes[t.slot] = std::max(slot_bytes[t.slot], like->tensor.ByteSize());
      }
    }
  }
  std::vector<std::size_t> slot_offset(slot_bytes.size());
  std::size_t cursor = Align256(plan->workspace_size_bytes);
  for (std::size_t s = 0; s < slot_bytes.size(); ++s) {
    slot_offset[s] = cursor;
    cursor += Align256(slot_bytes[s]);
  }
  for (const auto& op : ops) {
    for (const auto& c : op.candidates) {
      for (const auto& t : c.temporaries) {
        const bool seen = std::any_of(plan->allocations.begin(), plan->allocations.end(),
                                      [&](const Allocation& a) { return a.value_name == t.name; });
        if (seen) continue;
        plan->allocations.push_back(
            Allocation{t.name, graph.FindValue(t.like_value)->tensor.ByteSize(), slot_offset[t.slot], true, ""});
      }
    }
  }
  plan->workspace_size_bytes = Align256(cursor);
  return Status::OK();
}

}  // namespace

Status Compiler::Compile(const Model& model, const CompileOptions& options, ExecutablePlan* plan) const {
  if (plan == nullptr) return Status::InvalidArgument("ExecutablePlan output pointer is null");
  const bool cuda = IsCudaArtifactTarget(options.target);
  const std::string backend_name = CanonicalTargetName(options.target);
  if (options.allow_cpu_fallback && cuda) {
    return Status::Unsupported("CPU fallback inside a CUDA plan is not supported (no device transfer nodes)");
  }
  CUTRITON_RETURN_IF_ERROR(RegisterBuiltinBackends());

  ExecutablePlan result;
  result.mutable_graph() = model.graph();
  result.mutable_constants() = model.constants();
  CUTRITON_RETURN_IF_ERROR(ValidateProfiles(result.graph(), options.shape_profiles));
  if (!options.shape_profiles.empty()) {
    CUTRITON_RETURN_IF_ERROR(ApplyPoint(&result.mutable_graph(), options.shape_profiles.front(), Point::kOpt));
  }
  result.set_target(backend_name);
  result.set_enable_cuda_graph(options.enable_cuda_graph);
  result.set_enable_profiling(options.enable_profiling);
  TuningConfig& tuning = result.mutable_tuning_config();
  tuning.mode = options.tuning_mode;
  tuning.cache_dir = options.tuning_cache_dir;
  tuning.warmup_iterations = options.tuning_warmup_iterations;
  tuning.measurement_iterations = options.tuning_measurement_iterations;
  result.set_cuda_graph_cache_capacity(options.cuda_graph_cache_capacity);
  BackendOptions& backend_options = result.mutable_backend_options();
  backend_options.device = cuda ? Device::CUDA(options.device_id) : Device::CPU();
  backend_options.kernel_artifact_dir = options.kernel_artifact_dir;
  backend_options.kernel_artifact_paths = options.kernel_artifact_paths;
  if (backend_options.kernel_artifact_paths.empty() && !options.kernel_artifact_dir.empty()) {
    backend_options.kernel_artifact_paths.push_back(options.kernel_artifact_dir);
  }
  if (tuning.cache_dir.empty() && !backend_options.kernel_artifact_paths.empty()) {
    tuning.cache_dir = backend_options.kernel_artifact_paths.front() + "/tuning";
  }
  for (const auto& entry : result.graph().values()) {
    if (entry.second.is_constant && result.constants().count(entry.first) == 0) {
      return Status::InvalidArgument("constant value has no tensor data: " + entry.first);
    }
  }

  PassManager passes = CreateCompilePasses(options.enable_transformer_fusions, options.enable_residual_fusion);
  CUTRITON_RETURN_IF_ERROR(passes.Run(&result.mutable_graph()));

  if (cuda) {
    std::vector<std::pair<std::string, TensorDesc>> retagged;
    for (const auto& entry : result.graph().values()) {
      if (entry.second.tensor.dtype == DataType::kUnknown) continue;
      TensorDesc desc = entry.second.tensor;
      desc.device_type = DeviceType::kCUDA;
      desc.device_id = options.device_id;
      retagged.emplace_back(entry.first, std::move(desc));
    }
    for (auto& entry : retagged) {
      CUTRITON_RETURN_IF_ERROR(result.mutable_graph().SetValueDesc(entry.first, std::move(entry.second)));
    }
  }

  auto backend = KernelRegistry::Global().GetBackend(backend_name);
  if (backend == nullptr) return Status::NotFound("target backend is not registered: " + options.target);

  ArtifactRepository artifacts;
  const ArtifactRepository* repository = nullptr;
  if (cuda) {
    CUTRITON_RETURN_IF_ERROR(artifacts.Load(backend_options.kernel_artifact_paths));
    repository = &artifacts;
  }
  KernelCatalog catalog(repository);
  const LoweringContext lowering{&result.graph(), &result.backend_options(), repository,
                                 repository == nullptr ? nullptr : &catalog};
  for (const auto& node : result.graph().nodes()) {
    PlanOp op{node.id(), node.name(), node.op_type(), backend->name(), node.inputs(), node.outputs(), {}, 0};
    const Status lowered = backend->Lower(node, lowering, &op.candidates);
    if (!lowered.ok()) {
      // Missing packs keep their NotFound code so callers can tell them apart.
      if (lowered.code() == ErrorCode::kNotFound) return lowered;
      return Status::Unsupported("node " + node.name() + " (" + node.op_type() +
                                 ") is not supported by " + options.target + ": " + lowered.message());
    }
    if (op.candidates.empty()) return Status::Internal("backend produced no candidate for " + node.name());
    for (std::size_t i = 0; i < op.candidates.size(); ++i) {
      if (op.candidates[i].is_default) {
        op.selected_candidate = i;
        break;
      }
    }
    result.mutable_ops().push_back(std::move(op));
  }

  MemoryPlanner planner;
  if (options.shape_profiles.empty()) {
    CUTRITON_RETURN_IF_ERROR(planner.Plan(result.graph(), &result.mutable_memory_plan()));
    CUTRITON_RETURN_IF_ERROR(AddCandidateTemporaries(result.graph(), result.ops(), &result.mutable_memory_plan()));
  } else {
    for (const auto& profile : options.shape_profiles) {
      ProfilePlan pp;
      pp.profile = profile;
      CUTRITON_RETURN_IF_ERROR(ResolveAt(result.graph(), profile, Point::kMin, &pp.min_graph));
      CUTRITON_RETURN_IF_ERROR(ResolveAt(result.graph(), profile, Point::kOpt, &pp.opt_graph));
      CUTRITON_RETURN_IF_ERROR(ResolveAt(result.graph(), profile, Point::kMax, &pp.max_graph));
      CUTRITON_RETURN_IF_ERROR(planner.Plan(pp.max_graph, &pp.max_memory_plan));
      CUTRITON_RETURN_IF_ERROR(AddCandidateTemporaries(pp.max_graph, result.ops(), &pp.max_memory_plan));
      result.mutable_profile_plans().push_back(std::move(pp));
    }
    result.mutable_memory_plan() = result.profile_plans().front().max_memory_plan;
  }
  *plan = std::move(result);
  return Status::OK();
}

Status BuildEngine(const Model& model, const CompileOptions& options, std::unique_ptr<Engine>* engine) {
  if (engine == nullptr) return Status::InvalidArgument("Engine output pointer is null");
  ExecutablePlan plan;
  CUTRITON_RETURN_IF_ERROR(Compiler{}.Compile(model, options, &plan));
  *engine = std::make_unique<Engine>(std::move(plan));
  return Status::OK();
}

}  // namespace cutriton
