// Engine and ExecutionContext.
//
// Engine holds the compiled plan and, in EngineState, what every context of
// it shares: device copies of the constants (plus their prepacked forms,
// derived once at upload) and the CUDA module cache. Both are created on
// first use, once.
//
// An ExecutionContext keeps all of its mutable state in one Session. Staleness
// is tracked with epochs instead of a flag per stage: changing the shape
// profile or an input shape bumps the layout epoch, binding a graph-boundary
// tensor bumps the binding epoch, pinning a candidate bumps the choice epoch.
// Each stage remembers the epochs it was built at and rebuilds when they
// moved:
//
//   tensor table   layout, binding   constants + workspace views + bindings
//   selection      layout, choice    default / pinned / tuned candidate per op
//   kernels        layout, choice    OpKernels of the selected candidates
//
// RunAsync on a CUDA plan enqueues the kernels directly, or — with CUDA
// Graphs on — replays the graph captured for the current launch fingerprint
// (profile, workspace, bound addresses and shapes, selected candidates) from
// an LRU GraphCache. Kernels get the DeviceSession's error word as their
// runtime scratch; Synchronize reports an expired bounded wait from it.

#include "cutriton/runtime/engine.h"

#include <algorithm>
#include <mutex>
#include <optional>
#include <variant>

#include "../backend/prepack.h"
#include "../cuda_driver.h"
#include "cutriton/core/buffer.h"
#include "cutriton/ir/pass.h"
#include "device_session.h"
#include "tuner.h"

namespace cutriton {

// ---- shared engine state ---------------------------------------------------------

class EngineState {
 public:
  explicit EngineState(ExecutablePlan compiled) : plan(std::move(compiled)) {}

  bool on_cuda() const { return plan.backend_options().device.type == DeviceType::kCUDA; }
  int device_id() const { return plan.backend_options().device.id; }

  // Device constants (host tensors as they are for CPU plans).
  Status Constants(const std::unordered_map<std::string, Tensor>** out) {
    std::call_once(constants_once_, [this]() { constants_status_ = BuildConstants(); });
    *out = &constants_;
    return constants_status_;
  }

  Status Modules(std::shared_ptr<CudaModuleCache>* out) {
    if (on_cuda()) {
      std::call_once(modules_once_, [this]() { modules_status_ = CreateCudaModuleCache(device_id(), &modules_); });
    }
    *out = modules_;
    return modules_status_;
  }

  std::size_t module_count() const { return LoadedModuleCount(modules_); }

  const ExecutablePlan plan;

 private:
  Status Place(const std::string& name, TensorDesc desc, const void* host_bytes) {
    desc.device_type = DeviceType::kCUDA;
    desc.device_id = device_id();
    std::shared_ptr<Buffer> buffer;
    CUTRITON_RETURN_IF_ERROR(Buffer::AllocateCuda(desc.ByteSize(), device_id(), &buffer));
    CUTRITON_RETURN_IF_ERROR(buffer->CopyFromHost(host_bytes, desc.ByteSize()));
    constants_[name] = Tensor(std::move(desc), std::move(buffer));
    return Status::OK();
  }

  static const std::uint8_t* HostBytes(const Tensor& t) {
    return static_cast<const std::uint8_t*>(t.buffer()->data()) + t.byte_offset();
  }

  Status BuildConstants() {
    for (const auto& [name, host] : plan.constants()) {
      const ValueDesc* value = plan.graph().FindValue(name);
      if (value == nullptr || !value->is_constant) {
        return Status::Internal("plan constant '" + name + "' is not a constant of the graph");
      }
      if (!on_cuda()) {
        constants_.emplace(name, host);
        continue;
      }
      CUTRITON_RETURN_IF_ERROR(Place(name, value->tensor, HostBytes(host)));
    }
    if (!on_cuda()) return Status::OK();
    // Prepacked forms named by kernel arguments of any candidate.
    for (const PlanOp& op : plan.ops()) {
      for (const ExecutionCandidate& candidate : op.candidates) {
        for (const PlanStep& step : candidate.steps) {
          const auto* invocation = std::get_if<KernelInvocation>(&step);
          if (invocation == nullptr) continue;
          for (const auto& argument : invocation->artifact.arguments) {
            const std::string& transform = argument.source.prepack;
            if (transform.empty()) continue;
            const auto slot = static_cast<std::size_t>(argument.source.index);
            if (slot >= invocation->inputs.size()) {
              return Status::Internal("kernel " + invocation->artifact.kernel_id + ": prepack argument '" +
                                      argument.name + "' names input " + std::to_string(slot));
            }
            const std::string& base = invocation->inputs[slot];
            const std::string derived = PrepackedName(base, transform);
            if (constants_.count(derived) != 0) continue;
            const auto host = plan.constants().find(base);
            if (host == plan.constants().end()) {
              return Status::InvalidArgument("prepack '" + transform + "' needs a constant, '" + base + "' is not one");
            }
            TensorDesc packed_desc;
            std::vector<std::uint8_t> packed;
            CUTRITON_RETURN_IF_ERROR(RunPrepack(transform, plan.graph().FindValue(base)->tensor,
                                                HostBytes(host->second), &packed_desc, &packed));
            CUTRITON_RETURN_IF_ERROR(Place(derived, std::move(packed_desc), packed.data()));
          }
        }
      }
    }
    return Status::OK();
  }

  std::once_flag constants_once_;
  Status constants_status_;
  std::unordered_map<std::string, Tensor> constants_;
  std::once_flag modules_once_;
  Status modules_status_;
  std::shared_ptr<CudaModuleCache> modules_;
};

Engine::Engine(ExecutablePlan plan) : state_(std::make_shared<EngineState>(std::move(plan))) {}

const ExecutablePlan& Engine::plan() const { return state_->plan; }

std::unique_ptr<ExecutionContext> Engine::CreateExecutionContext() const {
  return std::make_unique<ExecutionContext>(state_);
}

// ---- per-context session -----------------------------------------------------------

struct ExecutionContext::Session {
  // Shapes.
  int profile{-1};
  std::unordered_map<std::string, std::vector<int64_t>> input_shapes;
  Graph resolved;
  bool resolved_ok{false};

  // Epochs (see the file comment) and what each stage was built at.
  std::uint64_t layout{1}, binding{1}, choice{1};
  std::pair<std::uint64_t, std::uint64_t> table_at{0, 0};
  std::pair<std::uint64_t, std::uint64_t> selection_at{0, 0};
  std::pair<std::uint64_t, std::uint64_t> kernels_at{0, 0};

  std::unordered_map<std::string, Tensor> bound;    // graph inputs / outputs given by the caller
  std::unordered_map<std::string, Tensor> tensors;  // everything a kernel may look up
  std::shared_ptr<Buffer> workspace;
  std::unordered_map<std::size_t, std::size_t> pins;
  std::vector<std::size_t> chosen;
  std::vector<std::vector<std::unique_ptr<OpKernel>>> kernels;
  std::vector<char> timed;  // per op: profiled with events (has a kernel launch)

  Profiler profiler;
  bool pending{false};
  CUstream stream{nullptr};
  std::unique_ptr<runtime::DeviceSession> device;
  std::unique_ptr<runtime::GraphCache> graphs;

  const Graph& graph(const ExecutablePlan& plan) const { return resolved_ok ? resolved : plan.graph(); }
  void ShapesChanged() {
    ++layout;
    bound.clear();
    tensors.clear();
  }
};

namespace {

Status CheckBinding(const std::string& name, const TensorDesc& want, const Tensor& tensor) {
  CUTRITON_RETURN_IF_ERROR(tensor.desc().Validate());
  const std::string where = "binding '" + name + "': ";
  if (!tensor.defined() || tensor.buffer()->empty()) return Status::InvalidArgument(where + "no buffer");
  const TensorDesc& got = tensor.desc();
  if (got.shape != want.shape || got.dtype != want.dtype || got.layout != want.layout) {
    return Status::InvalidArgument(where + "shape, dtype or layout differs from the plan");
  }
  if (got.device_type != want.device_type || got.device_id != want.device_id ||
      tensor.buffer()->device_type() != want.device_type || tensor.buffer()->device_id() != want.device_id) {
    return Status::InvalidArgument(where + "not on the plan's device");
  }
  const std::size_t capacity = tensor.buffer()->size_bytes();
  if (tensor.byte_offset() > capacity || want.ByteSize() > capacity - tensor.byte_offset()) {
    return Status::InvalidArgument(where + "the buffer is smaller than the tensor");
  }
  return Status::OK();
}

bool OnlyViews(const ExecutionCandidate& candidate) {
  return std::none_of(candidate.steps.begin(), candidate.steps.end(),
                      [](const PlanStep& s) { return std::holds_alternative<KernelInvocation>(s); });
}

}  // namespace

ExecutionContext::ExecutionContext(std::shared_ptr<EngineState> state)
    : state_(std::move(state)), session_(std::make_unique<Session>()) {
  // A plan with a single profile starts on it, at its opt shapes.
  if (state_ != nullptr && state_->plan.profile_plans().size() == 1) {
    const ProfilePlan& only = state_->plan.profile_plans().front();
    session_->profile = 0;
    session_->resolved = only.opt_graph;
    session_->resolved_ok = true;
    for (const auto& [input, range] : only.profile.inputs) session_->input_shapes[input] = range.opt;
  }
}

ExecutionContext::~ExecutionContext() {
  (void)Synchronize();
  if (session_->device != nullptr) (void)session_->device->MakeCurrent();
  session_->graphs.reset();
  session_->kernels.clear();
  session_->device.reset();
}

bool ExecutionContext::run_pending() const { return session_->pending; }
const Profiler& ExecutionContext::profiler() const { return session_->profiler; }
const std::unordered_map<std::string, Tensor>& ExecutionContext::tensors() const { return session_->tensors; }
const std::vector<std::size_t>& ExecutionContext::selected_candidates() const { return session_->chosen; }

std::size_t ExecutionContext::cached_cuda_graph_count() const {
  return session_->graphs == nullptr ? 0 : session_->graphs->size();
}

std::size_t ExecutionContext::loaded_cuda_module_count() const {
  return state_ == nullptr ? 0 : state_->module_count();
}

const Graph& ExecutionContext::ActiveGraph() const { return session_->graph(state_->plan); }

const MemoryPlan& ExecutionContext::ActiveMemoryPlan() const {
  const int p = session_->profile;
  return p >= 0 ? state_->plan.profile_plans().at(static_cast<std::size_t>(p)).max_memory_plan
                : state_->plan.memory_plan();
}

// ---- binding and shapes -------------------------------------------------------------

namespace {

Status CheckBoundary(bool pending, bool needs_resolve, const Graph& graph, const std::vector<std::string>& boundary,
                     const char* what, const std::string& name, const Tensor& tensor) {
  if (pending) return Status::RuntimeError("cannot bind '" + name + "' while a run is pending");
  if (needs_resolve) return Status::RuntimeError("call ResolveShapes before binding '" + name + "'");
  if (std::find(boundary.begin(), boundary.end(), name) == boundary.end()) {
    return Status::NotFound("'" + name + "' is not a graph " + what);
  }
  const ValueDesc* value = graph.FindValue(name);
  if (value == nullptr) return Status::NotFound("graph " + std::string(what) + " '" + name + "' has no description");
  return CheckBinding(name, value->tensor, tensor);
}

}  // namespace

Status ExecutionContext::BindInput(const std::string& name, Tensor tensor) {
  if (state_ == nullptr) return Status::InvalidArgument("BindInput: the context has no engine");
  const bool needs_resolve = !state_->plan.profile_plans().empty() && !session_->resolved_ok;
  CUTRITON_RETURN_IF_ERROR(
      CheckBoundary(session_->pending, needs_resolve, ActiveGraph(), ActiveGraph().inputs(), "input", name, tensor));
  // Visible through tensors() at once, before the next run rebuilds the table.
  session_->tensors[name] = tensor;
  session_->bound[name] = std::move(tensor);
  ++session_->binding;
  return Status::OK();
}

Status ExecutionContext::BindOutput(const std::string& name, Tensor tensor) {
  if (state_ == nullptr) return Status::InvalidArgument("BindOutput: the context has no engine");
  const bool needs_resolve = !state_->plan.profile_plans().empty() && !session_->resolved_ok;
  CUTRITON_RETURN_IF_ERROR(
      CheckBoundary(session_->pending, needs_resolve, ActiveGraph(), ActiveGraph().outputs(), "output", name, tensor));
  session_->tensors[name] = tensor;
  session_->bound[name] = std::move(tensor);
  ++session_->binding;
  return Status::OK();
}

Status ExecutionContext::SelectShapeProfile(const std::string& name) {
  Session& s = *session_;
  if (s.pending) return Status::RuntimeError("cannot switch shape profiles while a run is pending");
  const auto& plans = state_->plan.profile_plans();
  const auto it = std::find_if(plans.begin(), plans.end(), [&](const ProfilePlan& p) { return p.profile.name == name; });
  if (it == plans.end()) return Status::NotFound("no shape profile named '" + name + "'");
  s.profile = static_cast<int>(it - plans.begin());
  s.input_shapes.clear();
  for (const auto& [input, range] : it->profile.inputs) s.input_shapes[input] = range.opt;
  s.resolved = it->opt_graph;
  s.resolved_ok = true;
  s.ShapesChanged();
  s.workspace.reset();
  // Graphs captured for the old profile reference its workspace.
  if (s.graphs != nullptr) {
    if (s.device != nullptr) (void)s.device->MakeCurrent();
    s.graphs->Clear();
  }
  return Status::OK();
}

Status ExecutionContext::SetInputShape(const std::string& name, std::vector<int64_t> shape) {
  Session& s = *session_;
  if (s.pending) return Status::RuntimeError("cannot change input shapes while a run is pending");
  if (s.profile < 0) return Status::RuntimeError("SetInputShape needs a selected shape profile");
  const ShapeProfile& profile = state_->plan.profile_plans().at(static_cast<std::size_t>(s.profile)).profile;
  const auto range = profile.inputs.find(name);
  if (range == profile.inputs.end()) return Status::NotFound("'" + name + "' is not an input of the shape profile");
  const ShapeRange& r = range->second;
  if (shape.size() != r.min.size()) return Status::ShapeError("'" + name + "': rank differs from the profile");
  for (std::size_t axis = 0; axis < shape.size(); ++axis) {
    if (shape[axis] < r.min[axis] || shape[axis] > r.max[axis]) {
      return Status::ShapeError("'" + name + "': axis " + std::to_string(axis) + " is outside the profile's range");
    }
  }
  s.input_shapes[name] = std::move(shape);
  s.resolved_ok = false;
  s.ShapesChanged();
  return Status::OK();
}

Status ExecutionContext::ResolveShapes() {
  Session& s = *session_;
  if (s.profile < 0) return Status::RuntimeError("ResolveShapes needs a selected shape profile");
  Graph graph = state_->plan.profile_plans().at(static_cast<std::size_t>(s.profile)).opt_graph;
  for (const std::string& input : graph.inputs()) {
    const auto shape = s.input_shapes.find(input);
    if (shape == s.input_shapes.end()) return Status::InvalidArgument("no shape set for input '" + input + "'");
    graph.MutableValue(input)->tensor.shape = shape->second;
  }
  CUTRITON_RETURN_IF_ERROR(CreateShapeInferencePass()->Run(&graph));
  s.resolved = std::move(graph);
  s.resolved_ok = true;
  ++s.layout;
  return Status::OK();
}

const TensorDesc* ExecutionContext::GetResolvedTensorDesc(const std::string& name) const {
  if (!session_->resolved_ok) return nullptr;
  const ValueDesc* value = session_->resolved.FindValue(name);
  return value == nullptr ? nullptr : &value->tensor;
}

Status ExecutionContext::SelectCandidate(std::size_t op, std::size_t candidate) {
  if (session_->pending) return Status::RuntimeError("cannot pin a candidate while a run is pending");
  const auto& ops = state_->plan.ops();
  if (op >= ops.size()) return Status::InvalidArgument("SelectCandidate: op " + std::to_string(op) + " does not exist");
  if (candidate >= ops[op].candidates.size()) {
    return Status::InvalidArgument("SelectCandidate: op " + ops[op].node_name + " has no candidate " +
                                   std::to_string(candidate));
  }
  session_->pins[op] = candidate;
  ++session_->choice;
  return Status::OK();
}

// ---- preparation stages ---------------------------------------------------------------

Status ExecutionContext::PrepareTensors() {
  Session& s = *session_;
  if (s.table_at == std::make_pair(s.layout, s.binding)) return Status::OK();
  if (state_ == nullptr) return Status::InvalidArgument("the context has no engine");
  const std::unordered_map<std::string, Tensor>* constants = nullptr;
  CUTRITON_RETURN_IF_ERROR(state_->Constants(&constants));
  const MemoryPlan& memory = ActiveMemoryPlan();
  const Graph& graph = ActiveGraph();
  const Device& device = state_->plan.backend_options().device;
  if (memory.workspace_size_bytes > 0 && (s.workspace == nullptr || s.workspace->size_bytes() < memory.workspace_size_bytes)) {
    if (device.type == DeviceType::kCUDA) {
      CUTRITON_RETURN_IF_ERROR(Buffer::AllocateCuda(memory.workspace_size_bytes, device.id, &s.workspace));
    } else {
      s.workspace = Buffer::AllocateHost(memory.workspace_size_bytes);
    }
  }
  // Temporaries of unfused candidates are shaped like another value.
  std::unordered_map<std::string, std::string> temporary_like;
  for (const PlanOp& op : state_->plan.ops()) {
    for (const ExecutionCandidate& c : op.candidates) {
      for (const CandidateTemporary& t : c.temporaries) temporary_like.emplace(t.name, t.like_value);
    }
  }
  std::unordered_map<std::string, Tensor> table = *constants;
  for (const auto& [name, tensor] : s.bound) table[name] = tensor;
  for (const Allocation& a : memory.allocations) {
    const ValueDesc* value = graph.FindValue(a.value_name);
    if (value == nullptr) {
      const auto like = temporary_like.find(a.value_name);
      const ValueDesc* shape = like == temporary_like.end() ? nullptr : graph.FindValue(like->second);
      if (shape == nullptr) return Status::Internal("workspace entry '" + a.value_name + "' names no value");
      table[a.value_name] = Tensor(shape->tensor, s.workspace, a.offset);
      continue;
    }
    if (!a.alias_of.empty()) {
      // Allocations come in definition order, so a view's source (planned,
      // constant or bound) is already in the table.
      const auto source = table.find(a.alias_of);
      if (source == table.end()) return Status::Internal("view '" + a.value_name + "' has no source tensor");
      if (source->second.desc().ByteSize() != value->tensor.ByteSize()) {
        return Status::ShapeError("view '" + a.value_name + "' would change the byte size of '" + a.alias_of + "'");
      }
      table[a.value_name] = Tensor(value->tensor, source->second.buffer(), source->second.byte_offset());
      continue;
    }
    if (s.workspace == nullptr || a.offset > s.workspace->size_bytes() ||
        a.size_bytes > s.workspace->size_bytes() - a.offset) {
      return Status::Internal("workspace entry '" + a.value_name + "' lies outside the workspace");
    }
    table[a.value_name] = Tensor(value->tensor, s.workspace, a.offset);
  }
  s.tensors = std::move(table);
  s.table_at = {s.layout, s.binding};
  return Status::OK();
}

Status ExecutionContext::ValidateBindings() const {
  const Session& s = *session_;
  const Graph& graph = ActiveGraph();
  for (const std::string& name : graph.inputs()) {
    if (s.bound.count(name) == 0) return Status::InvalidArgument("graph input '" + name + "' is not bound");
  }
  for (const std::string& name : graph.outputs()) {
    if (s.bound.count(name) == 0) return Status::InvalidArgument("graph output '" + name + "' is not bound");
  }
  for (const Node& node : graph.nodes()) {
    for (const auto* names : {&node.inputs(), &node.outputs()}) {
      for (const std::string& name : *names) {
        if (s.tensors.count(name) == 0) {
          return Status::InvalidArgument("node '" + node.name() + "' uses '" + name + "', which has no tensor");
        }
      }
    }
  }
  return Status::OK();
}

Status ExecutionContext::PrepareTuning() {
  Session& s = *session_;
  if (s.selection_at == std::make_pair(s.layout, s.choice)) return Status::OK();
  const auto& ops = state_->plan.ops();
  std::vector<std::size_t> chosen(ops.size());
  for (std::size_t i = 0; i < ops.size(); ++i) {
    const auto pin = s.pins.find(i);
    chosen[i] = pin != s.pins.end() ? pin->second : ops[i].selected_candidate;
  }
  const TuningConfig& config = state_->plan.tuning_config();
  if (state_->on_cuda() && config.mode != TuningMode::kDisabled) {
    std::shared_ptr<CudaModuleCache> modules;
    CUTRITON_RETURN_IF_ERROR(state_->Modules(&modules));
    const int device_id = state_->device_id();
    const Graph& graph = ActiveGraph();
    for (std::size_t i = 0; i < ops.size(); ++i) {
      const PlanOp& op = ops[i];
      if (op.candidates.size() < 2 || s.pins.count(i) != 0) continue;
      const Node& node = graph.nodes().at(static_cast<std::size_t>(op.node_id));
      const std::string key = runtime::TuningFingerprint(op, node, graph, device_id);
      std::optional<std::string> cached;
      if (config.mode != TuningMode::kForceRetune) {
        cached = runtime::LoadTuningChoice(config.cache_dir, key);
        // UseCache also accepts a choice recorded at the profile's opt shapes.
        if (!cached && config.mode == TuningMode::kUseCache && s.profile >= 0) {
          const Graph& opt = state_->plan.profile_plans().at(static_cast<std::size_t>(s.profile)).opt_graph;
          cached = runtime::LoadTuningChoice(
              config.cache_dir,
              runtime::TuningFingerprint(op, opt.nodes().at(static_cast<std::size_t>(op.node_id)), opt, device_id));
        }
      }
      if (cached) {
        const auto match = std::find_if(op.candidates.begin(), op.candidates.end(),
                                        [&](const ExecutionCandidate& c) { return c.candidate_id == *cached; });
        if (match != op.candidates.end()) {
          chosen[i] = static_cast<std::size_t>(match - op.candidates.begin());
          continue;
        }
      }
      if (config.mode == TuningMode::kUseCache) continue;
      runtime::TuningTarget target;
      target.op = &op;
      target.node = &node;
      target.device_id = device_id;
      target.tensors = &s.tensors;
      target.error_word = s.device == nullptr ? nullptr : s.device->error_word_device();
      if (s.device != nullptr) target.take_device_error = [&s] { return s.device->TakeDeviceError(); };
      target.modules = modules;
      std::vector<double> medians;
      CUTRITON_RETURN_IF_ERROR(runtime::TuneCandidates(target, config, &chosen[i], &medians));
      CUTRITON_RETURN_IF_ERROR(runtime::StoreTuningChoice(config.cache_dir, key, op, chosen[i], medians));
    }
  }
  s.chosen = std::move(chosen);
  s.selection_at = {s.layout, s.choice};
  return Status::OK();
}

Status ExecutionContext::PrepareKernels() {
  Session& s = *session_;
  if (s.kernels_at == std::make_pair(s.layout, s.choice) && !s.kernels.empty()) return Status::OK();
  if (state_ == nullptr) return Status::InvalidArgument("the context has no engine");
  CUTRITON_RETURN_IF_ERROR(RegisterBuiltinBackends());
  std::shared_ptr<CudaModuleCache> modules;
  CUTRITON_RETURN_IF_ERROR(state_->Modules(&modules));
  const auto& ops = state_->plan.ops();
  if (s.chosen.size() != ops.size()) return Status::Internal("candidate selection has not run");
  const Graph& graph = ActiveGraph();
  const BackendOptions& options = state_->plan.backend_options();
  std::vector<std::vector<std::unique_ptr<OpKernel>>> built(ops.size());
  std::vector<char> timed(ops.size(), 0);
  for (std::size_t i = 0; i < ops.size(); ++i) {
    const PlanOp& op = ops[i];
    const std::shared_ptr<Backend> backend = KernelRegistry::Global().GetBackend(op.backend_name);
    if (backend == nullptr) return Status::NotFound("backend '" + op.backend_name + "' is not registered");
    if (s.chosen[i] >= op.candidates.size()) return Status::Internal("op " + op.node_name + ": candidate out of range");
    const ExecutionCandidate& candidate = op.candidates[s.chosen[i]];
    const Node& node = graph.nodes().at(static_cast<std::size_t>(op.node_id));
    const auto from_backend = [&]() -> Status {
      std::unique_ptr<OpKernel> kernel;
      CUTRITON_RETURN_IF_ERROR(backend->CreateKernel(node, graph, options, &kernel));
      if (kernel == nullptr) return Status::Internal("backend '" + op.backend_name + "' made no kernel for " + op.node_name);
      built[i].push_back(std::move(kernel));
      return Status::OK();
    };
    for (const PlanStep& step : candidate.steps) {
      if (const auto* invocation = std::get_if<KernelInvocation>(&step)) {
        std::unique_ptr<OpKernel> kernel;
        CUTRITON_RETURN_IF_ERROR(CreateInvocationKernel(*invocation, options.device.id, modules, &kernel));
        built[i].push_back(std::move(kernel));
      } else {
        CUTRITON_RETURN_IF_ERROR(from_backend());
      }
    }
    // A candidate without steps (CPU / plugin backends) runs the backend's kernel.
    if (candidate.steps.empty()) CUTRITON_RETURN_IF_ERROR(from_backend());
    timed[i] = !OnlyViews(candidate) && !candidate.steps.empty();
  }
  s.kernels = std::move(built);
  s.timed = std::move(timed);
  s.kernels_at = {s.layout, s.choice};
  return Status::OK();
}

void ExecutionContext::InvalidateCudaGraph() {
  if (session_->graphs == nullptr) return;
  if (session_->device != nullptr) (void)session_->device->MakeCurrent();
  session_->graphs->Clear();
}

// ---- running ----------------------------------------------------------------------------

Status ExecutionContext::Run() {
  CUTRITON_RETURN_IF_ERROR(RunAsync(nullptr));
  return Synchronize();
}

Status ExecutionContext::RunAsync(void* stream) {
  Session& s = *session_;
  if (s.pending) return Status::RuntimeError("RunAsync: the previous run has not been synchronised");
  CUTRITON_RETURN_IF_ERROR(PrepareTensors());
  CUTRITON_RETURN_IF_ERROR(ValidateBindings());
  const ExecutablePlan& plan = state_->plan;
  if (state_->on_cuda() && s.device == nullptr) {
    CUTRITON_RETURN_IF_ERROR(
        runtime::DeviceSession::Open(state_->device_id(), plan.ops().size(), plan.enable_profiling(), &s.device));
    s.graphs = std::make_unique<runtime::GraphCache>(plan.cuda_graph_cache_capacity());
  }
  CUTRITON_RETURN_IF_ERROR(PrepareTuning());
  CUTRITON_RETURN_IF_ERROR(PrepareKernels());
  const Graph& graph = ActiveGraph();

  if (!state_->on_cuda()) {
    // Host backends run synchronously; CPU timers record into the profiler.
    s.profiler.Clear();
    Profiler* profiler = plan.enable_profiling() ? &s.profiler : nullptr;
    for (std::size_t i = 0; i < s.kernels.size(); ++i) {
      const Node& node = graph.nodes().at(static_cast<std::size_t>(plan.ops()[i].node_id));
      KernelContext context{&node, &s.tensors, stream, profiler, nullptr};
      for (auto& kernel : s.kernels[i]) CUTRITON_RETURN_IF_ERROR(kernel->Compute(&context));
    }
    s.pending = true;
    return Status::OK();
  }

  const auto& api = drv::Get();
  CUTRITON_RETURN_IF_ERROR(s.device->MakeCurrent());
  s.stream = stream != nullptr ? static_cast<CUstream>(stream) : s.device->own_stream();
  const bool use_graphs = plan.enable_cuda_graph();
  const bool profiling = plan.enable_profiling() && s.device->has_events();
  void* error_word = s.device->error_word_device();

  const auto enqueue = [&]() -> Status {
    const auto mark = [&](CUevent event) {
      return use_graphs ? drv::Check(api.cuEventRecordWithFlags(event, s.stream, CU_EVENT_RECORD_EXTERNAL),
                                     "cuEventRecordWithFlags")
                        : drv::Check(api.cuEventRecord(event, s.stream), "cuEventRecord");
    };
    for (std::size_t i = 0; i < s.kernels.size(); ++i) {
      const Node& node = graph.nodes().at(static_cast<std::size_t>(plan.ops()[i].node_id));
      const bool timed = profiling && s.timed[i];
      if (timed) CUTRITON_RETURN_IF_ERROR(mark(s.device->op_start(i)));
      KernelContext context{&node, &s.tensors, s.stream, nullptr, error_word};
      for (auto& kernel : s.kernels[i]) CUTRITON_RETURN_IF_ERROR(kernel->Compute(&context));
      if (timed) CUTRITON_RETURN_IF_ERROR(mark(s.device->op_end(i)));
    }
    return Status::OK();
  };

  if (!use_graphs) {
    CUTRITON_RETURN_IF_ERROR(enqueue());
    s.pending = true;
    return Status::OK();
  }

  // Launch fingerprint: everything a captured graph has baked in.
  std::vector<std::uint64_t> fingerprint;
  const auto put = [&](std::uint64_t word) { fingerprint.push_back(word); };
  const auto put_tensor = [&](const Tensor& t) {
    put(reinterpret_cast<std::uintptr_t>(t.buffer()->data()));
    put(t.byte_offset());
    put(t.desc().shape.size());
    for (int64_t d : t.desc().shape) put(static_cast<std::uint64_t>(d));
  };
  put(static_cast<std::uint64_t>(s.profile + 1));
  put(reinterpret_cast<std::uintptr_t>(s.workspace == nullptr ? nullptr : s.workspace->data()));
  for (const std::string& name : graph.inputs()) put_tensor(s.bound.at(name));
  put(~0ull);
  for (const std::string& name : graph.outputs()) put_tensor(s.bound.at(name));
  put(~0ull);
  for (std::size_t c : s.chosen) put(c);

  CUgraphExec exec = nullptr;
  CUTRITON_RETURN_IF_ERROR(s.graphs->Acquire(fingerprint, s.stream, enqueue, &exec));
  CUTRITON_RETURN_IF_ERROR(drv::Check(api.cuGraphLaunch(exec, s.stream), "cuGraphLaunch"));
  s.pending = true;
  return Status::OK();
}

Status ExecutionContext::Synchronize() {
  Session& s = *session_;
  if (!s.pending) return Status::OK();
  s.pending = false;
  if (!state_->on_cuda()) return Status::OK();
  const auto& api = drv::Get();
  CUTRITON_RETURN_IF_ERROR(s.device->MakeCurrent());
  CUTRITON_RETURN_IF_ERROR(drv::Check(api.cuStreamSynchronize(s.stream), "cuStreamSynchronize"));
  CUTRITON_RETURN_IF_ERROR(s.device->TakeDeviceError());
  s.profiler.Clear();
  if (!state_->plan.enable_profiling()) return Status::OK();
  const auto& ops = state_->plan.ops();
  for (std::size_t i = 0; i < ops.size(); ++i) {
    float ms = 0.0f;
    if (s.device->has_events() && i < s.timed.size() && s.timed[i]) {
      CUTRITON_RETURN_IF_ERROR(
          drv::Check(api.cuEventElapsedTime(&ms, s.device->op_start(i), s.device->op_end(i)), "cuEventElapsedTime"));
    }
    s.profiler.Record(ops[i].node_name, ops[i].backend_name, static_cast<double>(ms));
  }
  return Status::OK();
}

}  // namespace cutriton
