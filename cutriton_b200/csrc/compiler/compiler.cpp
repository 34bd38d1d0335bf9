// Model -> ExecutablePlan.
//
// A compilation is a CompileJob that runs a fixed list of stages over one
// ExecutablePlan under construction:
//
//   Request     reject option combinations the backend cannot honour
//   Seed        copy graph + constants, record runtime settings
//   Profiles    check every shape profile; pin the graph at the first
//               profile's opt point
//   Passes      shape inference, DCE and the fusion passes
//   Placement   CUDA targets: every typed value lives on the plan's device
//   Lowering    each node -> execution candidates (the default selected)
//   Workspace   memory plan: static, or per profile at its max point, plus
//               shared slots for the temporaries of unfused candidates
//
// Dynamic shapes are handled by ProfileSpace: it validates the ranges and
// produces the graph concretised at a profile's min / opt / max point.
// Whether a target is a CUDA artifact backend is a property of the target
// ("cuda_sm100", alias "cuda_triton"), not a string comparison spread over the
// stages.

#include "cutriton/compiler/compiler.h"

#include <algorithm>
#include <functional>
#include <map>

#include "cutriton/backend/backend.h"
#include "cutriton/ir/pass.h"
#include "cutriton/runtime/memory_planner.h"

namespace cutriton {
namespace {

constexpr std::size_t kSlotAlign = 256;

std::size_t SlotRound(std::size_t bytes) { return (bytes + kSlotAlign - 1) & ~(kSlotAlign - 1); }

// ---- dynamic shapes -------------------------------------------------------------

enum class Corner { kMin, kOpt, kMax };

class ProfileSpace {
 public:
  explicit ProfileSpace(const std::vector<ShapeProfile>& profiles) : profiles_(profiles) {}

  // Every profile is named and gives each graph input a range of one rank
  // with 0 < min <= opt <= max on every axis.
  Status Check(const Graph& graph) const {
    for (const ShapeProfile& profile : profiles_) {
      if (profile.name.empty()) return Status::InvalidArgument("shape profile without a name");
      for (const std::string& input : graph.inputs()) {
        const auto range = profile.inputs.find(input);
        const std::string where = "shape profile '" + profile.name + "', input '" + input + "': ";
        if (range == profile.inputs.end()) return Status::InvalidArgument(where + "no range given");
        const ShapeRange& r = range->second;
        const std::size_t rank = r.min.size();
        if (rank == 0 || r.opt.size() != rank || r.max.size() != rank) {
          return Status::ShapeError(where + "min, opt and max must have the same nonzero rank");
        }
        for (std::size_t axis = 0; axis < rank; ++axis) {
          if (!(0 < r.min[axis] && r.min[axis] <= r.opt[axis] && r.opt[axis] <= r.max[axis])) {
            return Status::ShapeError(where + "axis " + std::to_string(axis) + " breaks 0 < min <= opt <= max");
          }
        }
      }
    }
    return Status::OK();
  }

  // Sets every graph input to the profile's shape at `corner`.
  static Status Pin(Graph* graph, const ShapeProfile& profile, Corner corner) {
    for (const std::string& input : graph->inputs()) {
      const ValueDesc* value = graph->FindValue(input);
      if (value == nullptr) return Status::NotFound("graph input '" + input + "' has no value");
      const ShapeRange& r = profile.inputs.at(input);
      TensorDesc desc = value->tensor;
      desc.shape = corner == Corner::kMin ? r.min : (corner == Corner::kMax ? r.max : r.opt);
      CUTRITON_RETURN_IF_ERROR(graph->SetValueDesc(input, std::move(desc)));
    }
    return Status::OK();
  }

  // The compiled graph re-inferred at one corner of a profile.
  static Status Concretise(const Graph& compiled, const ShapeProfile& profile, Corner corner, Graph* out) {
    Graph graph = compiled;
    CUTRITON_RETURN_IF_ERROR(Pin(&graph, profile, corner));
    CUTRITON_RETURN_IF_ERROR(CreateShapeInferencePass()->Run(&graph));
    *out = std::move(graph);
    return Status::OK();
  }

 private:
  const std::vector<ShapeProfile>& profiles_;
};

// ---- candidate temporaries ------------------------------------------------------

// Unfused candidates keep intermediate tensors in numbered slots; a slot is
// shared by every temporary that names it, sized for the largest, and the
// slots are appended after the planned workspace.
Status AppendTemporarySlots(const Graph& graph, const std::vector<PlanOp>& ops, MemoryPlan* plan) {
  std::map<std::size_t, std::size_t> slot_bytes;
  std::vector<std::pair<const CandidateTemporary*, std::size_t>> users;  // temporary, its bytes
  for (const PlanOp& op : ops) {
    for (const ExecutionCandidate& candidate : op.candidates) {
      for (const CandidateTemporary& t : candidate.temporaries) {
        const ValueDesc* like = graph.FindValue(t.like_value);
        const std::size_t bytes = like == nullptr ? 0 : like->tensor.ByteSize();
        if (bytes == 0) {
          return Status::ShapeError("temporary '" + t.name + "' of " + op.node_name +
                                    " copies the shape of a value with no static size");
        }
        std::size_t& slot = slot_bytes[t.slot];
        slot = std::max(slot, bytes);
        users.emplace_back(&t, bytes);
      }
    }
  }
  std::map<std::size_t, std::size_t> slot_offset;
  std::size_t end = SlotRound(plan->workspace_size_bytes);
  for (const auto& [slot, bytes] : slot_bytes) {
    slot_offset[slot] = end;
    end += SlotRound(bytes);
  }
  std::vector<std::string> listed;
  for (const auto& [t, bytes] : users) {
    if (std::find(listed.begin(), listed.end(), t->name) != listed.end()) continue;
    listed.push_back(t->name);
    plan->allocations.push_back(Allocation{t->name, bytes, slot_offset.at(t->slot), true, ""});
  }
  plan->workspace_size_bytes = SlotRound(end);
  return Status::OK();
}

// ---- the job ----------------------------------------------------------------------

class CompileJob {
 public:
  CompileJob(const Model& model, const CompileOptions& options)
      : model_(model), options_(options), cuda_(IsCudaArtifactTarget(options.target)),
        backend_name_(CanonicalTargetName(options.target)), profiles_(options.shape_profiles) {}

  Status Run(ExecutablePlan* out) {
    const std::vector<Status (CompileJob::*)()> stages = {
        &CompileJob::Request, &CompileJob::Seed,     &CompileJob::Profiles, &CompileJob::Passes,
        &CompileJob::Placement, &CompileJob::Lowering, &CompileJob::Workspace};
    for (auto stage : stages) CUTRITON_RETURN_IF_ERROR((this->*stage)());
    *out = std::move(plan_);
    return Status::OK();
  }

 private:
  Status Request() {
    if (options_.allow_cpu_fallback && cuda_) {
      return Status::Unsupported("allow_cpu_fallback: a CUDA plan has no device-transfer nodes to fall back with");
    }
    return RegisterBuiltinBackends();
  }

  Status Seed() {
    plan_.mutable_graph() = model_.graph();
    plan_.mutable_constants() = model_.constants();
    for (const auto& [name, value] : plan_.graph().values()) {
      if (value.is_constant && plan_.constants().count(name) == 0) {
        return Status::InvalidArgument("constant '" + name + "' has no tensor data in the model");
      }
    }
    plan_.set_target(backend_name_);
    plan_.set_enable_cuda_graph(options_.enable_cuda_graph);
    plan_.set_enable_profiling(options_.enable_profiling);
    plan_.set_cuda_graph_cache_capacity(options_.cuda_graph_cache_capacity);

    BackendOptions& backend = plan_.mutable_backend_options();
    backend.device = cuda_ ? Device::CUDA(options_.device_id) : Device::CPU();
    backend.kernel_artifact_dir = options_.kernel_artifact_dir;
    backend.kernel_artifact_paths = options_.kernel_artifact_paths;
    if (backend.kernel_artifact_paths.empty() && !backend.kernel_artifact_dir.empty()) {
      backend.kernel_artifact_paths = {backend.kernel_artifact_dir};
    }

    TuningConfig& tuning = plan_.mutable_tuning_config();
    tuning.mode = options_.tuning_mode;
    tuning.warmup_iterations = options_.tuning_warmup_iterations;
    tuning.measurement_iterations = options_.tuning_measurement_iterations;
    // Without an explicit cache directory the tuning cache sits next to the
    // first kernel pack.
    tuning.cache_dir = !options_.tuning_cache_dir.empty() || backend.kernel_artifact_paths.empty()
                           ? options_.tuning_cache_dir
                           : backend.kernel_artifact_paths.front() + "/tuning";
    return Status::OK();
  }

  Status Profiles() {
    CUTRITON_RETURN_IF_ERROR(profiles_.Check(plan_.graph()));
    if (options_.shape_profiles.empty()) return Status::OK();
    return ProfileSpace::Pin(&plan_.mutable_graph(), options_.shape_profiles.front(), Corner::kOpt);
  }

  Status Passes() {
    return CreateCompilePasses(options_.enable_transformer_fusions, options_.enable_residual_fusion)
        .Run(&plan_.mutable_graph());
  }

  Status Placement() {
    if (!cuda_) return Status::OK();
    Graph& graph = plan_.mutable_graph();
    std::vector<std::string> typed;
    for (const auto& [name, value] : graph.values()) {
      if (value.tensor.dtype != DataType::kUnknown) typed.push_back(name);
    }
    for (const std::string& name : typed) {
      ValueDesc* value = graph.MutableValue(name);
      value->tensor.device_type = DeviceType::kCUDA;
      value->tensor.device_id = options_.device_id;
    }
    return Status::OK();
  }

  Status Lowering() {
    const std::shared_ptr<Backend> backend = KernelRegistry::Global().GetBackend(backend_name_);
    if (backend == nullptr) return Status::NotFound("no backend is registered for target '" + options_.target + "'");
    if (cuda_) CUTRITON_RETURN_IF_ERROR(artifacts_.Load(plan_.backend_options().kernel_artifact_paths));
    const ArtifactRepository* repository = cuda_ ? &artifacts_ : nullptr;
    KernelCatalog catalog(repository);
    const LoweringContext context{&plan_.graph(), &plan_.backend_options(), repository,
                                  repository == nullptr ? nullptr : &catalog};
    std::vector<PlanOp> ops;
    ops.reserve(plan_.graph().nodes().size());
    for (const Node& node : plan_.graph().nodes()) {
      PlanOp op;
      op.node_id = node.id();
      op.node_name = node.name();
      op.op_type = node.op_type();
      op.backend_name = backend->name();
      op.inputs = node.inputs();
      op.outputs = node.outputs();
      const Status lowered = backend->Lower(node, context, &op.candidates);
      // A missing pack keeps NotFound so callers can tell it from an
      // unsupported node.
      if (lowered.code() == ErrorCode::kNotFound) return lowered;
      if (!lowered.ok()) {
        return Status::Unsupported(options_.target + " cannot run node '" + node.name() + "' (" + node.op_type() +
                                   "): " + lowered.message());
      }
      if (op.candidates.empty()) return Status::Internal("lowering of '" + node.name() + "' produced no candidate");
      const auto chosen = std::find_if(op.candidates.begin(), op.candidates.end(),
                                       [](const ExecutionCandidate& c) { return c.is_default; });
      op.selected_candidate = chosen == op.candidates.end() ? 0 : chosen - op.candidates.begin();
      ops.push_back(std::move(op));
    }
    plan_.mutable_ops() = std::move(ops);
    return Status::OK();
  }

  Status Workspace() {
    const MemoryPlanner planner;
    if (options_.shape_profiles.empty()) {
      MemoryPlan& memory = plan_.mutable_memory_plan();
      CUTRITON_RETURN_IF_ERROR(planner.Plan(plan_.graph(), &memory));
      return AppendTemporarySlots(plan_.graph(), plan_.ops(), &memory);
    }
    // One workspace per profile, sized at its max point (every shape the
    // profile admits fits in it).
    for (const ShapeProfile& profile : options_.shape_profiles) {
      ProfilePlan pp;
      pp.profile = profile;
      CUTRITON_RETURN_IF_ERROR(ProfileSpace::Concretise(plan_.graph(), profile, Corner::kMin, &pp.min_graph));
      CUTRITON_RETURN_IF_ERROR(ProfileSpace::Concretise(plan_.graph(), profile, Corner::kOpt, &pp.opt_graph));
      CUTRITON_RETURN_IF_ERROR(ProfileSpace::Concretise(plan_.graph(), profile, Corner::kMax, &pp.max_graph));
      CUTRITON_RETURN_IF_ERROR(planner.Plan(pp.max_graph, &pp.max_memory_plan));
      CUTRITON_RETURN_IF_ERROR(AppendTemporarySlots(pp.max_graph, plan_.ops(), &pp.max_memory_plan));
      plan_.mutable_profile_plans().push_back(std::move(pp));
    }
    plan_.mutable_memory_plan() = plan_.profile_plans().front().max_memory_plan;
    return Status::OK();
  }

  const Model& model_;
  const CompileOptions& options_;
  const bool cuda_;
  const std::string backend_name_;
  ProfileSpace profiles_;
  ArtifactRepository artifacts_;
  ExecutablePlan plan_;
};

}  // namespace

Status Compiler::Compile(const Model& model, const CompileOptions& options, ExecutablePlan* plan) const {
  if (plan == nullptr) return Status::InvalidArgument("Compiler::Compile: no ExecutablePlan to write");
  return CompileJob(model, options).Run(plan);
}

Status BuildEngine(const Model& model, const CompileOptions& options, std::unique_ptr<Engine>* engine) {
  if (engine == nullptr) return Status::InvalidArgument("BuildEngine: no Engine pointer to write");
  ExecutablePlan plan;
  CUTRITON_RETURN_IF_ERROR(Compiler{}.Compile(model, options, &plan));
  *engine = std::make_unique<Engine>(std::move(plan));
  return Status::OK();
}

}  // namespace cutriton
