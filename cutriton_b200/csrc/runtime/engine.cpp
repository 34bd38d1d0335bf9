// Engine / ExecutionContext: binding, shape profiles, workspace views,
// candidate tuning with an on-disk cache, CUDA Graph capture with an LRU of
// instantiated graphs, per-op event profiling and the device error block.
//
// Semantics follow the reference runtime (src/runtime/engine.cpp): binding
// validation 86-111/426-472, profiles 486-571, PrepareTensors 593-668,
// PrepareKernels 670-723, PrepareTuning 725-891 (FNV-1a tuning key 215-295,
// atomic JSON cache 297-335), RunAsync 925-1079 and Synchronize 1081-1119.
// Added here: constant prepacking at upload, and the error block — a small
// pinned, device-mapped host buffer bound to each kernel's first
// runtime_reserved parameter; kernels with bounded spin-waits record an
// expired wait there instead of hanging, and Synchronize reports it.

#include "cutriton/runtime/engine.h"

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <filesystem>
#include <fstream>
#include <iomanip>
#include <limits>
#include <mutex>
#include <optional>
#include <sstream>
#include <type_traits>
#include <variant>

#include "../backend/prepack.h"
#include "../cuda_driver.h"
#include "cutriton/core/buffer.h"
#include "cutriton/ir/pass.h"

namespace cutriton {
namespace {

bool Contains(const std::vector<std::string>& list, const std::string& name) {
  return std::find(list.begin(), list.end(), name) != list.end();
}

// IEEE binary16 -> binary32 (exact).
float HalfToFloat(std::uint16_t h) {
  const std::uint32_t sign = std::uint32_t(h & 0x8000u) << 16;
  const std::uint32_t exp = (h >> 10) & 0x1Fu;
  std::uint32_t man = h & 0x3FFu;
  std::uint32_t bits;
  if (exp == 0x1Fu) {
    bits = sign | 0x7F800000u | (man << 13);
  } else if (exp != 0) {
    bits = sign | ((exp + 112u) << 23) | (man << 13);
  } else if (man == 0) {
    bits = sign;
  } else {
    int e = -1;
    do { man <<= 1; ++e; } while ((man & 0x400u) == 0);
    bits = sign | (std::uint32_t(112 - e) << 23) | ((man & 0x3FFu) << 13);
  }
  float f;
  std::memcpy(&f, &bits, sizeof f);
  return f;
}

Status ValidateBoundTensor(const std::string& name, const TensorDesc& expected, const Tensor& tensor) {
  CUTRITON_RETURN_IF_ERROR(tensor.desc().Validate());
  if (!tensor.defined() || tensor.buffer()->empty()) {
    return Status::InvalidArgument("tensor buffer is not defined: " + name);
  }
  const TensorDesc& actual = tensor.desc();
  if (actual.shape != expected.shape || actual.dtype != expected.dtype ||
      actual.layout != expected.layout || actual.device_type != expected.device_type ||
      actual.device_id != expected.device_id) {
    return Status::InvalidArgument("tensor description does not match the plan: " + name);
  }
  if (tensor.buffer()->device_type() != expected.device_type ||
      tensor.buffer()->device_id() != expected.device_id) {
    return Status::InvalidArgument("tensor buffer is on the wrong device: " + name);
  }
  if (tensor.byte_offset() > tensor.buffer()->size_bytes() ||
      expected.ByteSize() > tensor.buffer()->size_bytes() - tensor.byte_offset()) {
    return Status::InvalidArgument("tensor buffer is too small: " + name);
  }
  return Status::OK();
}

Status CopyAsFloat(const Tensor& tensor, std::vector<float>* out) {
  const auto count = static_cast<std::size_t>(tensor.desc().NumElements());
  out->assign(count, 0.0f);
  if (tensor.desc().dtype == DataType::kFloat32) {
    return tensor.buffer()->CopyToHost(out->data(), tensor.desc().ByteSize(), tensor.byte_offset());
  }
  if (tensor.desc().dtype == DataType::kFloat16) {
    std::vector<std::uint16_t> half(count);
    CUTRITON_RETURN_IF_ERROR(tensor.buffer()->CopyToHost(half.data(), tensor.desc().ByteSize(), tensor.byte_offset()));
    for (std::size_t i = 0; i < count; ++i) (*out)[i] = HalfToFloat(half[i]);
    return Status::OK();
  }
  return Status::Unsupported("tuning comparison supports float32/float16 only");
}

struct EventPair {
  CUevent start{nullptr};
  CUevent end{nullptr};
  bool timed{false};
};

struct GraphEntry {
  std::string key;
  CUgraph graph{nullptr};
  CUgraphExec exec{nullptr};
  std::uint64_t last_used{0};
};

// Layout of the error block shared with kernels (see kernels/common.cuh).
struct ErrorBlock {
  std::uint32_t code;     // 0 = no error
  std::uint32_t site;     // kernel-defined location of the expired wait
  std::uint32_t block;    // linear CTA index that gave up
  std::uint32_t reserved[13];
};

struct CudaState {
  CUdevice device{};
  CUcontext context{nullptr};
  CUstream owned_stream{nullptr};
  CUstream active_stream{nullptr};
  std::vector<GraphEntry> graphs;
  std::uint64_t clock{0};
  std::vector<EventPair> events;
  ErrorBlock* error_host{nullptr};
  CUdeviceptr error_device{0};
};

void DestroyGraphs(CudaState* s) {
  const auto& api = drv::Get();
  for (auto& g : s->graphs) {
    if (g.exec != nullptr) api.cuGraphExecDestroy(g.exec);
    if (g.graph != nullptr) api.cuGraphDestroy(g.graph);
  }
  s->graphs.clear();
}

void DestroyCudaState(CudaState* s) {
  if (s == nullptr) return;
  const auto& api = drv::Get();
  if (s->context != nullptr) api.cuCtxSetCurrent(s->context);
  DestroyGraphs(s);
  for (auto& e : s->events) {
    if (e.start != nullptr) api.cuEventDestroy(e.start);
    if (e.end != nullptr) api.cuEventDestroy(e.end);
  }
  if (s->owned_stream != nullptr) api.cuStreamDestroy(s->owned_stream);
  if (s->error_host != nullptr) api.cuMemFreeHost(s->error_host);
  if (s->context != nullptr) api.cuDevicePrimaryCtxRelease(s->device);
  delete s;
}

Status InitializeCudaState(CudaState* s, int device_id, std::size_t ops, bool profiling) {
  CUTRITON_RETURN_IF_ERROR(drv::RetainPrimaryContext(device_id, &s->device, &s->context));
  const auto& api = drv::Get();
  CUTRITON_RETURN_IF_ERROR(drv::Check(api.cuStreamCreate(&s->owned_stream, CU_STREAM_NON_BLOCKING), "cuStreamCreate"));
  void* host = nullptr;
  CUTRITON_RETURN_IF_ERROR(drv::Check(
      api.cuMemHostAlloc(&host, sizeof(ErrorBlock), CU_MEMHOSTALLOC_DEVICEMAP | CU_MEMHOSTALLOC_PORTABLE),
      "cuMemHostAlloc"));
  s->error_host = static_cast<ErrorBlock*>(host);
  std::memset(s->error_host, 0, sizeof(ErrorBlock));
  CUTRITON_RETURN_IF_ERROR(drv::Check(api.cuMemHostGetDevicePointer(&s->error_device, host, 0),
                                      "cuMemHostGetDevicePointer"));
  s->events.resize(ops);
  if (profiling) {
    for (auto& e : s->events) {
      CUTRITON_RETURN_IF_ERROR(drv::Check(api.cuEventCreate(&e.start, CU_EVENT_DEFAULT), "cuEventCreate"));
      CUTRITON_RETURN_IF_ERROR(drv::Check(api.cuEventCreate(&e.end, CU_EVENT_DEFAULT), "cuEventCreate"));
    }
  }
  return Status::OK();
}

std::string Hex64(std::uint64_t v) {
  std::ostringstream out;
  out << std::hex << std::setw(16) << std::setfill('0') << v;
  return out.str();
}

// Tuning cache key: FNV-1a 64 over the op, its tensors (dtype, layout,
// shape), its attributes, every candidate's kernel identity and binary hash,
// and the device (SM, UUID) and driver version.
std::string TuningKey(const PlanOp& op, const Node& node, const Graph& graph, int device_id) {
  std::ostringstream m;
  m << op.op_type << '|' << device_id;
  auto tensors = [&](const char* role, const std::vector<std::string>& names) {
    for (const auto& name : names) {
      m << '|' << role << ':' << name;
      if (const ValueDesc* v = graph.FindValue(name)) {
        m << ':' << static_cast<int>(v->tensor.dtype) << ':' << v->tensor.layout;
        for (int64_t d : v->tensor.shape) m << ':' << d;
      }
    }
  };
  tensors("input", op.inputs);
  tensors("output", op.outputs);
  std::vector<std::string> keys;
  for (const auto& a : node.attributes()) keys.push_back(a.first);
  std::sort(keys.begin(), keys.end());
  for (const auto& k : keys) {
    const Attribute& attr = node.attributes().at(k);
    m << "|attribute:" << k << ':' << attr.index();
    std::visit([&](const auto& v) {
      using T = std::decay_t<decltype(v)>;
      if constexpr (std::is_same_v<T, std::vector<int64_t>> || std::is_same_v<T, std::vector<double>>) {
        for (const auto& x : v) m << ':' << x;
      } else {
        m << ':' << v;
      }
    }, attr);
  }
  for (const auto& c : op.candidates) {
    m << '|' << c.candidate_id;
    for (const auto& step : c.steps) {
      if (const auto* inv = std::get_if<KernelInvocation>(&step)) {
        const KernelArtifact& a = inv->artifact;
        m << "|pack:" << a.pack_name << ':' << a.pack_version << "|kernel:" << a.kernel_id << ':'
          << a.kernel_version << ':' << a.variant_id << "|abi:" << a.abi_schema_version
          << "|generator:" << a.generator_version << "|binary:" << a.sha256;
      } else {
        m << "|view";
      }
    }
  }
  const auto& api = drv::Get();
  CUdevice device{};
  if (api.available && api.cuDeviceGet(&device, device_id) == CUDA_SUCCESS) {
    int major = 0, minor = 0;
    CUuuid uuid{};
    api.cuDeviceGetUuid(&uuid, device);
    api.cuDeviceGetAttribute(&major, CU_DEVICE_ATTRIBUTE_COMPUTE_CAPABILITY_MAJOR, device);
    api.cuDeviceGetAttribute(&minor, CU_DEVICE_ATTRIBUTE_COMPUTE_CAPABILITY_MINOR, device);
    m << "|sm:" << major << minor << "|uuid:" << std::hex;
    for (char b : uuid.bytes) m << static_cast<int>(static_cast<unsigned char>(b));
    m << std::dec;
  }
  int driver = 0;
  if (api.available) api.cuDriverGetVersion(&driver);
  m << "|driver:" << driver;
  std::uint64_t h = 14695981039346656037ull;
  for (unsigned char c : m.str()) {
    h ^= c;
    h *= 1099511628211ull;
  }
  return Hex64(h);
}

std::optional<std::string> ReadTuningChoice(const std::filesystem::path& path) {
  std::ifstream in(path);
  if (!in) return std::nullopt;
  std::ostringstream text;
  text << in.rdbuf();
  const std::string s = text.str();
  const std::string marker = "\"candidate_id\": \"";
  const auto begin = s.find(marker);
  if (begin == std::string::npos) return std::nullopt;
  const auto start = begin + marker.size();
  const auto end = s.find('"', start);
  if (end == std::string::npos) return std::nullopt;
  return s.substr(start, end - start);
}

// Writes to a temporary file and renames it over the target (atomic publish).
Status WriteTuningChoice(const std::filesystem::path& path, const std::string& key,
                         const std::string& candidate_id, double median_ms) {
  std::error_code error;
  std::filesystem::create_directories(path.parent_path(), error);
  if (error) return Status::RuntimeError("cannot create the tuning cache directory: " + error.message());
  const std::string temporary = path.string() + ".tmp";
  {
    std::ofstream out(temporary, std::ios::trunc);
    out << "{\n  \"schema_version\": 1,\n  \"tuning_key\": \"" << key << "\",\n  \"candidate_id\": \""
        << candidate_id << "\",\n  \"median_ms\": " << median_ms << "\n}\n";
    if (!out) return Status::RuntimeError("cannot write the tuning cache");
  }
  std::filesystem::rename(temporary, path, error);
  if (error) {
    std::filesystem::remove(path, error);
    error.clear();
    std::filesystem::rename(temporary, path, error);
  }
  return error ? Status::RuntimeError("cannot publish the tuning cache: " + error.message()) : Status::OK();
}

std::optional<std::size_t> CandidateIndex(const PlanOp& op, const std::string& id) {
  for (std::size_t i = 0; i < op.candidates.size(); ++i) {
    if (op.candidates[i].candidate_id == id) return i;
  }
  return std::nullopt;
}

}  // namespace

class EngineState {
 public:
  explicit EngineState(ExecutablePlan p) : plan(std::move(p)) {}

  Status InitializeConstants() {
    std::call_once(constants_once_, [&]() { constants_status_ = UploadConstants(); });
    return constants_status_;
  }

  Status InitializeModuleCache() {
    if (plan.backend_options().device.type != DeviceType::kCUDA) return Status::OK();
    std::call_once(cache_once_, [&]() {
      cache_status_ = CreateCudaModuleCache(plan.backend_options().device.id, &module_cache);
    });
    return cache_status_;
  }

  ExecutablePlan plan;
  std::unordered_map<std::string, Tensor> device_constants;
  std::shared_ptr<CudaModuleCache> module_cache;

 private:
  Status Upload(const std::string& name, const TensorDesc& desc, const void* bytes) {
    std::shared_ptr<Buffer> buffer;
    CUTRITON_RETURN_IF_ERROR(Buffer::AllocateCuda(desc.ByteSize(), plan.backend_options().device.id, &buffer));
    CUTRITON_RETURN_IF_ERROR(buffer->CopyFromHost(bytes, desc.ByteSize()));
    device_constants[name] = Tensor(desc, std::move(buffer));
    return Status::OK();
  }

  Status UploadConstants() {
    const bool cpu = plan.backend_options().device.type == DeviceType::kCPU;
    for (const auto& entry : plan.constants()) {
      const ValueDesc* value = plan.graph().FindValue(entry.first);
      if (value == nullptr || !value->is_constant) {
        return Status::Internal("plan constant is missing from the graph: " + entry.first);
      }
      if (cpu) {
        device_constants.emplace(entry.first, entry.second);
        continue;
      }
      const Tensor& source = entry.second;
      const auto* bytes = static_cast<const std::uint8_t*>(source.buffer()->data()) + source.byte_offset();
      CUTRITON_RETURN_IF_ERROR(Upload(entry.first, value->tensor, bytes));
    }
    if (cpu) return Status::OK();
    // Derived constants for every prepacked argument of every candidate.
    for (const auto& op : plan.ops()) {
      for (const auto& candidate : op.candidates) {
        for (const auto& step : candidate.steps) {
          const auto* inv = std::get_if<KernelInvocation>(&step);
          if (inv == nullptr) continue;
          for (const auto& arg : inv->artifact.arguments) {
            if (arg.source.prepack.empty()) continue;
            const auto index = static_cast<std::size_t>(arg.source.index);
            if (index >= inv->inputs.size()) return Status::Internal("prepack argument index is invalid");
            const std::string& base = inv->inputs[index];
            const std::string derived = PrepackedName(base, arg.source.prepack);
            if (device_constants.count(derived) != 0) continue;
            const auto found = plan.constants().find(base);
            if (found == plan.constants().end()) {
              return Status::InvalidArgument("prepacked argument does not bind a constant: " + base);
            }
            const Tensor& host = found->second;
            TensorDesc desc = plan.graph().FindValue(base)->tensor;
            TensorDesc out_desc;
            std::vector<std::uint8_t> out_bytes;
            CUTRITON_RETURN_IF_ERROR(RunPrepack(
                arg.source.prepack, desc,
                static_cast<const std::uint8_t*>(host.buffer()->data()) + host.byte_offset(), &out_desc,
                &out_bytes));
            out_desc.device_type = DeviceType::kCUDA;
            out_desc.device_id = plan.backend_options().device.id;
            CUTRITON_RETURN_IF_ERROR(Upload(derived, out_desc, out_bytes.data()));
          }
        }
      }
    }
    return Status::OK();
  }

  std::once_flag constants_once_;
  Status constants_status_;
  std::once_flag cache_once_;
  Status cache_status_;
};

Engine::Engine(ExecutablePlan plan) : state_(std::make_shared<EngineState>(std::move(plan))) {}

const ExecutablePlan& Engine::plan() const { return state_->plan; }

std::unique_ptr<ExecutionContext> Engine::CreateExecutionContext() const {
  return std::make_unique<ExecutionContext>(state_);
}

ExecutionContext::ExecutionContext(std::shared_ptr<EngineState> state) : state_(std::move(state)) {
  if (state_ != nullptr && state_->plan.profile_plans().size() == 1) {
    selected_profile_ = 0;
    const ProfilePlan& pp = state_->plan.profile_plans().front();
    resolved_graph_ = pp.opt_graph;
    shapes_resolved_ = true;
    for (const auto& entry : pp.profile.inputs) input_shapes_[entry.first] = entry.second.opt;
  }
}

ExecutionContext::~ExecutionContext() {
  (void)Synchronize();
  DestroyCudaState(static_cast<CudaState*>(cuda_state_));
}

const Graph& ExecutionContext::ActiveGraph() const {
  return shapes_resolved_ ? resolved_graph_ : state_->plan.graph();
}

const MemoryPlan& ExecutionContext::ActiveMemoryPlan() const {
  if (selected_profile_ >= 0) {
    return state_->plan.profile_plans().at(static_cast<std::size_t>(selected_profile_)).max_memory_plan;
  }
  return state_->plan.memory_plan();
}

Status ExecutionContext::BindInput(const std::string& name, Tensor tensor) {
  if (state_ == nullptr) return Status::InvalidArgument("ExecutionContext has no engine state");
  if (run_pending_) return Status::RuntimeError("cannot bind a tensor while a run is pending");
  if (!state_->plan.profile_plans().empty() && !shapes_resolved_) {
    return Status::RuntimeError("ResolveShapes must be called before binding");
  }
  const Graph& graph = ActiveGraph();
  if (!Contains(graph.inputs(), name)) return Status::NotFound("name is not a graph input: " + name);
  const ValueDesc* value = graph.FindValue(name);
  if (value == nullptr) return Status::NotFound("graph input description is missing: " + name);
  CUTRITON_RETURN_IF_ERROR(ValidateBoundTensor(name, value->tensor, tensor));
  tensors_[name] = std::move(tensor);
  tensors_prepared_ = false;
  return Status::OK();
}

Status ExecutionContext::BindOutput(const std::string& name, Tensor tensor) {
  if (state_ == nullptr) return Status::InvalidArgument("ExecutionContext has no engine state");
  if (run_pending_) return Status::RuntimeError("cannot bind a tensor while a run is pending");
  if (!state_->plan.profile_plans().empty() && !shapes_resolved_) {
    return Status::RuntimeError("ResolveShapes must be called before binding");
  }
  const Graph& graph = ActiveGraph();
  if (!Contains(graph.outputs(), name)) return Status::NotFound("name is not a graph output: " + name);
  const ValueDesc* value = graph.FindValue(name);
  if (value == nullptr) return Status::NotFound("graph output description is missing: " + name);
  CUTRITON_RETURN_IF_ERROR(ValidateBoundTensor(name, value->tensor, tensor));
  tensors_[name] = std::move(tensor);
  tensors_prepared_ = false;
  return Status::OK();
}

Status ExecutionContext::SelectShapeProfile(const std::string& name) {
  if (run_pending_) return Status::RuntimeError("cannot change the profile while a run is pending");
  const auto& profiles = state_->plan.profile_plans();
  const auto found = std::find_if(profiles.begin(), profiles.end(),
                                  [&](const ProfilePlan& p) { return p.profile.name == name; });
  if (found == profiles.end()) return Status::NotFound("ShapeProfile is not defined: " + name);
  selected_profile_ = static_cast<int>(found - profiles.begin());
  input_shapes_.clear();
  for (const auto& entry : found->profile.inputs) input_shapes_[entry.first] = entry.second.opt;
  resolved_graph_ = found->opt_graph;
  shapes_resolved_ = true;
  tensors_.clear();
  workspace_.reset();
  tensors_prepared_ = false;
  kernels_.clear();
  kernels_prepared_ = false;
  tuning_prepared_ = false;
  InvalidateCudaGraph();
  return Status::OK();
}

Status ExecutionContext::SetInputShape(const std::string& name, std::vector<int64_t> shape) {
  if (run_pending_) return Status::RuntimeError("cannot change a shape while a run is pending");
  if (selected_profile_ < 0) return Status::RuntimeError("select a ShapeProfile before setting shapes");
  const ShapeProfile& profile =
      state_->plan.profile_plans().at(static_cast<std::size_t>(selected_profile_)).profile;
  const auto range = profile.inputs.find(name);
  if (range == profile.inputs.end()) return Status::NotFound("name is not a profiled graph input: " + name);
  if (shape.size() != range->second.min.size()) {
    return Status::ShapeError("input shape rank does not match the profile: " + name);
  }
  for (std::size_t a = 0; a < shape.size(); ++a) {
    if (shape[a] < range->second.min[a] || shape[a] > range->second.max[a]) {
      return Status::ShapeError("input shape is outside the profile range: " + name);
    }
  }
  input_shapes_[name] = std::move(shape);
  shapes_resolved_ = false;
  tensors_.clear();
  tensors_prepared_ = false;
  kernels_.clear();
  kernels_prepared_ = false;
  tuning_prepared_ = false;
  return Status::OK();
}

Status ExecutionContext::ResolveShapes() {
  if (selected_profile_ < 0) return Status::RuntimeError("select a ShapeProfile before resolving shapes");
  const ProfilePlan& pp = state_->plan.profile_plans().at(static_cast<std::size_t>(selected_profile_));
  Graph graph = pp.opt_graph;
  for (const auto& input : graph.inputs()) {
    const auto shape = input_shapes_.find(input);
    if (shape == input_shapes_.end()) return Status::InvalidArgument("input shape is not set: " + input);
    TensorDesc desc = graph.FindValue(input)->tensor;
    desc.shape = shape->second;
    CUTRITON_RETURN_IF_ERROR(graph.SetValueDesc(input, std::move(desc)));
  }
  CUTRITON_RETURN_IF_ERROR(CreateShapeInferencePass()->Run(&graph));
  resolved_graph_ = std::move(graph);
  shapes_resolved_ = true;
  return Status::OK();
}

const TensorDesc* ExecutionContext::GetResolvedTensorDesc(const std::string& name) const {
  if (!shapes_resolved_) return nullptr;
  const ValueDesc* v = resolved_graph_.FindValue(name);
  return v == nullptr ? nullptr : &v->tensor;
}

std::size_t ExecutionContext::cached_cuda_graph_count() const {
  const auto* s = static_cast<const CudaState*>(cuda_state_);
  return s == nullptr ? 0 : s->graphs.size();
}

std::size_t ExecutionContext::loaded_cuda_module_count() const {
  return state_ == nullptr ? 0 : LoadedModuleCount(state_->module_cache);
}

Status ExecutionContext::PrepareTensors() {
  if (tensors_prepared_) return Status::OK();
  if (state_ == nullptr) return Status::InvalidArgument("ExecutionContext has no engine state");
  CUTRITON_RETURN_IF_ERROR(state_->InitializeConstants());
  for (const auto& entry : state_->device_constants) tensors_[entry.first] = entry.second;
  const MemoryPlan& plan = ActiveMemoryPlan();
  const BackendOptions& options = state_->plan.backend_options();
  if (plan.workspace_size_bytes != 0 &&
      (workspace_ == nullptr || workspace_->size_bytes() < plan.workspace_size_bytes)) {
    if (options.device.type == DeviceType::kCUDA) {
      CUTRITON_RETURN_IF_ERROR(Buffer::AllocateCuda(plan.workspace_size_bytes, options.device.id, &workspace_));
    } else {
      workspace_ = Buffer::AllocateHost(plan.workspace_size_bytes);
    }
  }
  const Graph& graph = ActiveGraph();
  for (const auto& a : plan.allocations) {
    const ValueDesc* value = graph.FindValue(a.value_name);
    if (value == nullptr) {
      // Candidate temporary: shaped like its `like_value`.
      const ValueDesc* like = nullptr;
      for (const auto& op : state_->plan.ops()) {
        for (const auto& c : op.candidates) {
          for (const auto& t : c.temporaries) {
            if (t.name == a.value_name) like = graph.FindValue(t.like_value);
          }
        }
        if (like != nullptr) break;
      }
      if (like == nullptr) return Status::Internal("allocation references an unknown value: " + a.value_name);
      tensors_[a.value_name] = Tensor(like->tensor, workspace_, a.offset);
      continue;
    }
    if (!a.alias_of.empty()) {
      const auto source = tensors_.find(a.alias_of);
      if (source == tensors_.end()) return Status::Internal("alias source tensor is missing: " + a.alias_of);
      if (value->tensor.ByteSize() != source->second.desc().ByteSize()) {
        return Status::ShapeError("alias changes the byte size: " + a.value_name);
      }
      tensors_[a.value_name] = Tensor(value->tensor, source->second.buffer(), source->second.byte_offset());
      continue;
    }
    if (workspace_ == nullptr || a.offset > workspace_->size_bytes() ||
        a.size_bytes > workspace_->size_bytes() - a.offset) {
      return Status::Internal("allocation exceeds the workspace: " + a.value_name);
    }
    tensors_[a.value_name] = Tensor(value->tensor, workspace_, a.offset);
  }
  tensors_prepared_ = true;
  return Status::OK();
}

Status ExecutionContext::PrepareKernels() {
  if (kernels_prepared_) return Status::OK();
  if (state_ == nullptr) return Status::InvalidArgument("ExecutionContext has no engine state");
  CUTRITON_RETURN_IF_ERROR(RegisterBuiltinBackends());
  CUTRITON_RETURN_IF_ERROR(state_->InitializeModuleCache());
  const auto& ops = state_->plan.ops();
  if (selected_candidates_.size() != ops.size()) return Status::Internal("tuning selections are not prepared");
  kernels_.clear();
  for (std::size_t i = 0; i < ops.size(); ++i) {
    const PlanOp& op = ops[i];
    auto backend = KernelRegistry::Global().GetBackend(op.backend_name);
    if (backend == nullptr) return Status::NotFound("backend is not registered: " + op.backend_name);
    const Node& node = ActiveGraph().nodes().at(static_cast<std::size_t>(op.node_id));
    if (selected_candidates_[i] >= op.candidates.size()) {
      return Status::Internal("selected execution candidate is out of range");
    }
    const ExecutionCandidate& candidate = op.candidates[selected_candidates_[i]];
    std::vector<std::unique_ptr<OpKernel>> group;
    for (const auto& step : candidate.steps) {
      std::unique_ptr<OpKernel> kernel;
      if (const auto* inv = std::get_if<KernelInvocation>(&step)) {
        CUTRITON_RETURN_IF_ERROR(CreateInvocationKernel(*inv, state_->plan.backend_options().device.id,
                                                        state_->module_cache, &kernel));
      } else {
        CUTRITON_RETURN_IF_ERROR(backend->CreateKernel(node, ActiveGraph(), state_->plan.backend_options(), &kernel));
      }
      if (kernel == nullptr) return Status::Internal("backend returned a null OpKernel");
      group.push_back(std::move(kernel));
    }
    if (group.empty()) {
      std::unique_ptr<OpKernel> kernel;
      CUTRITON_RETURN_IF_ERROR(backend->CreateKernel(node, ActiveGraph(), state_->plan.backend_options(), &kernel));
      if (kernel == nullptr) return Status::Internal("backend returned a null OpKernel");
      group.push_back(std::move(kernel));
    }
    kernels_.push_back(std::move(group));
  }
  kernels_prepared_ = true;
  return Status::OK();
}

Status ExecutionContext::PrepareTuning() {
  if (tuning_prepared_) return Status::OK();
  const auto& ops = state_->plan.ops();
  selected_candidates_.clear();
  for (const auto& op : ops) selected_candidates_.push_back(op.selected_candidate);
  for (const auto& pin : pinned_candidates_) selected_candidates_[pin.first] = pin.second;
  const TuningConfig& config = state_->plan.tuning_config();
  if (state_->plan.backend_options().device.type != DeviceType::kCUDA || config.mode == TuningMode::kDisabled) {
    tuning_prepared_ = true;
    return Status::OK();
  }
  CUTRITON_RETURN_IF_ERROR(state_->InitializeModuleCache());
  const auto& api = drv::Get();
  const int device_id = state_->plan.backend_options().device.id;
  for (std::size_t i = 0; i < ops.size(); ++i) {
    const PlanOp& op = ops[i];
    if (op.candidates.size() < 2 || pinned_candidates_.count(i) != 0) continue;
    const Node& node = ActiveGraph().nodes().at(static_cast<std::size_t>(op.node_id));
    const std::string key = TuningKey(op, node, ActiveGraph(), device_id);
    const std::filesystem::path cache_file = std::filesystem::path(config.cache_dir) / (key + ".json");
    if (config.mode != TuningMode::kForceRetune) {
      if (const auto cached = ReadTuningChoice(cache_file)) {
        if (const auto index = CandidateIndex(op, *cached)) {
          selected_candidates_[i] = *index;
          continue;
        }
      }
      if (config.mode == TuningMode::kUseCache && selected_profile_ >= 0) {
        const Graph& opt = state_->plan.profile_plans().at(static_cast<std::size_t>(selected_profile_)).opt_graph;
        const std::string opt_key = TuningKey(op, opt.nodes().at(static_cast<std::size_t>(op.node_id)), opt, device_id);
        if (const auto cached = ReadTuningChoice(std::filesystem::path(config.cache_dir) / (opt_key + ".json"))) {
          if (const auto index = CandidateIndex(op, *cached)) {
            selected_candidates_[i] = *index;
            continue;
          }
        }
      }
    }
    if (config.mode == TuningMode::kUseCache) continue;

    CUstream stream{};
    CUevent start{}, end{};
    CUTRITON_RETURN_IF_ERROR(drv::Check(api.cuStreamCreate(&stream, CU_STREAM_NON_BLOCKING), "cuStreamCreate"));
    CUTRITON_RETURN_IF_ERROR(drv::Check(api.cuEventCreate(&start, CU_EVENT_DEFAULT), "cuEventCreate"));
    CUTRITON_RETURN_IF_ERROR(drv::Check(api.cuEventCreate(&end, CU_EVENT_DEFAULT), "cuEventCreate"));
    struct Cleanup {
      CUstream s; CUevent a, b;
      ~Cleanup() {
        const auto& d = drv::Get();
        d.cuEventDestroy(a);
        d.cuEventDestroy(b);
        d.cuStreamDestroy(s);
      }
    } cleanup{stream, start, end};
    auto* cuda = static_cast<CudaState*>(cuda_state_);
    void* scratch = cuda == nullptr ? nullptr : reinterpret_cast<void*>(cuda->error_device);
    double best_ms = std::numeric_limits<double>::infinity();
    std::size_t best = op.selected_candidate;
    std::vector<float> reference;
    // The default candidate runs first and is the numerical reference (it is
    // always eligible); intermediate inputs may hold anything during tuning,
    // so elements where it is not finite are not compared.
    std::vector<std::size_t> order{op.selected_candidate};
    for (std::size_t c = 0; c < op.candidates.size(); ++c) {
      if (c != op.selected_candidate) order.push_back(c);
    }
    for (const std::size_t c : order) {
      std::vector<std::unique_ptr<OpKernel>> kernels;
      for (const auto& step : op.candidates[c].steps) {
        const auto* inv = std::get_if<KernelInvocation>(&step);
        if (inv == nullptr) continue;
        std::unique_ptr<OpKernel> kernel;
        CUTRITON_RETURN_IF_ERROR(CreateInvocationKernel(*inv, device_id, state_->module_cache, &kernel));
        kernels.push_back(std::move(kernel));
      }
      if (kernels.empty()) continue;
      KernelContext ctx{&node, &tensors_, stream, nullptr, scratch};
      for (int w = 0; w < config.warmup_iterations; ++w) {
        for (auto& k : kernels) CUTRITON_RETURN_IF_ERROR(k->Compute(&ctx));
      }
      CUTRITON_RETURN_IF_ERROR(drv::Check(api.cuStreamSynchronize(stream), "cuStreamSynchronize"));
      std::vector<float> produced;
      CUTRITON_RETURN_IF_ERROR(CopyAsFloat(tensors_.at(op.outputs.front()), &produced));
      if (reference.empty()) {
        reference = produced;
      } else {
        // Numerically different candidates are never chosen.
        const float rel = tensors_.at(op.outputs.front()).desc().dtype == DataType::kFloat16 ? 1e-2f : 1e-4f;
        bool same = true;
        for (std::size_t e = 0; e < produced.size() && same; ++e) {
          if (!std::isfinite(reference[e])) continue;
          const float tol = rel + rel * std::fabs(reference[e]);
          same = std::isfinite(produced[e]) && std::fabs(produced[e] - reference[e]) <= tol;
        }
        if (!same) continue;
      }
      std::vector<float> samples;
      for (int r = 0; r < config.measurement_iterations; ++r) {
        CUTRITON_RETURN_IF_ERROR(drv::Check(api.cuEventRecord(start, stream), "cuEventRecord"));
        for (auto& k : kernels) CUTRITON_RETURN_IF_ERROR(k->Compute(&ctx));
        CUTRITON_RETURN_IF_ERROR(drv::Check(api.cuEventRecord(end, stream), "cuEventRecord"));
        CUTRITON_RETURN_IF_ERROR(drv::Check(api.cuEventSynchronize(end), "cuEventSynchronize"));
        float ms = 0.0f;
        CUTRITON_RETURN_IF_ERROR(drv::Check(api.cuEventElapsedTime(&ms, start, end), "cuEventElapsedTime"));
        samples.push_back(ms);
      }
      if (samples.empty()) continue;
      std::sort(samples.begin(), samples.end());
      const double median = samples[samples.size() / 2];
      if (median < best_ms) {
        best_ms = median;
        best = c;
      }
    }
    if (!std::isfinite(best_ms)) return Status::RuntimeError("no numerically valid tuning candidate for " + op.node_name);
    selected_candidates_[i] = best;
    CUTRITON_RETURN_IF_ERROR(WriteTuningChoice(cache_file, key, op.candidates[best].candidate_id, best_ms));
  }
  tuning_prepared_ = true;
  return Status::OK();
}

Status ExecutionContext::SelectCandidate(std::size_t op, std::size_t candidate) {
  if (run_pending_) return Status::RuntimeError("cannot select a candidate while a run is pending");
  const auto& ops = state_->plan.ops();
  if (op >= ops.size()) return Status::InvalidArgument("plan op index is out of range");
  if (candidate >= ops[op].candidates.size()) return Status::InvalidArgument("candidate index is out of range");
  pinned_candidates_[op] = candidate;
  tuning_prepared_ = false;
  kernels_prepared_ = false;
  kernels_.clear();
  return Status::OK();
}

Status ExecutionContext::ValidateBindings() const {
  const Graph& graph = ActiveGraph();
  for (const auto& name : graph.inputs()) {
    if (tensors_.count(name) == 0) return Status::InvalidArgument("graph input is not bound: " + name);
  }
  for (const auto& name : graph.outputs()) {
    if (tensors_.count(name) == 0) return Status::InvalidArgument("graph output is not bound: " + name);
  }
  for (const auto& node : graph.nodes()) {
    for (const auto& name : node.inputs()) {
      if (tensors_.count(name) == 0) return Status::InvalidArgument("node input tensor is missing: " + name);
    }
    for (const auto& name : node.outputs()) {
      if (tensors_.count(name) == 0) return Status::InvalidArgument("node output tensor is missing: " + name);
    }
  }
  return Status::OK();
}

Status ExecutionContext::Run() {
  CUTRITON_RETURN_IF_ERROR(RunAsync(nullptr));
  return Synchronize();
}

Status ExecutionContext::RunAsync(void* stream) {
  if (run_pending_) return Status::RuntimeError("a run is already pending");
  CUTRITON_RETURN_IF_ERROR(PrepareTensors());
  CUTRITON_RETURN_IF_ERROR(ValidateBindings());
  const bool use_cuda = state_->plan.backend_options().device.type == DeviceType::kCUDA;
  if (use_cuda && cuda_state_ == nullptr) {
    auto* created = new CudaState();
    const Status status = InitializeCudaState(created, state_->plan.backend_options().device.id,
                                              state_->plan.ops().size(), state_->plan.enable_profiling());
    if (!status.ok()) {
      DestroyCudaState(created);
      return status;
    }
    cuda_state_ = created;
  }
  CUTRITON_RETURN_IF_ERROR(PrepareTuning());
  CUTRITON_RETURN_IF_ERROR(PrepareKernels());

  if (!use_cuda) {
    profiler_.Clear();
    for (std::size_t i = 0; i < kernels_.size(); ++i) {
      const PlanOp& op = state_->plan.ops()[i];
      const Node& node = ActiveGraph().nodes().at(static_cast<std::size_t>(op.node_id));
      KernelContext ctx{&node, &tensors_, stream, state_->plan.enable_profiling() ? &profiler_ : nullptr, nullptr};
      for (auto& kernel : kernels_[i]) CUTRITON_RETURN_IF_ERROR(kernel->Compute(&ctx));
    }
    run_pending_ = true;
    return Status::OK();
  }

  auto* cuda = static_cast<CudaState*>(cuda_state_);
  const auto& api = drv::Get();
  CUTRITON_RETURN_IF_ERROR(drv::Check(api.cuCtxSetCurrent(cuda->context), "cuCtxSetCurrent"));
  cuda->active_stream = stream == nullptr ? cuda->owned_stream : reinterpret_cast<CUstream>(stream);
  const bool graphs = state_->plan.enable_cuda_graph();
  const bool profiling = state_->plan.enable_profiling();
  void* scratch = reinterpret_cast<void*>(cuda->error_device);

  auto enqueue = [&]() -> Status {
    auto record = [&](CUevent e) {
      return graphs ? drv::Check(api.cuEventRecordWithFlags(e, cuda->active_stream, CU_EVENT_RECORD_EXTERNAL),
                                 "cuEventRecordWithFlags")
                    : drv::Check(api.cuEventRecord(e, cuda->active_stream), "cuEventRecord");
    };
    for (std::size_t i = 0; i < kernels_.size(); ++i) {
      const PlanOp& op = state_->plan.ops()[i];
      const Node& node = ActiveGraph().nodes().at(static_cast<std::size_t>(op.node_id));
      EventPair& events = cuda->events[i];
      events.timed = profiling && node.op_type() != "Flatten";
      if (events.timed) CUTRITON_RETURN_IF_ERROR(record(events.start));
      KernelContext ctx{&node, &tensors_, cuda->active_stream, nullptr, scratch};
      for (auto& kernel : kernels_[i]) CUTRITON_RETURN_IF_ERROR(kernel->Compute(&ctx));
      if (events.timed) CUTRITON_RETURN_IF_ERROR(record(events.end));
    }
    return Status::OK();
  };

  if (!graphs) {
    CUTRITON_RETURN_IF_ERROR(enqueue());
    run_pending_ = true;
    return Status::OK();
  }

  std::ostringstream k;
  k << "profile:" << selected_profile_ << "|workspace:" << (workspace_ ? workspace_->data() : nullptr);
  for (const auto& name : ActiveGraph().inputs()) {
    const Tensor& t = tensors_.at(name);
    k << "|in:" << name << ':' << t.buffer()->data() << ':' << t.byte_offset();
    for (int64_t d : t.desc().shape) k << ':' << d;
  }
  for (const auto& name : ActiveGraph().outputs()) {
    const Tensor& t = tensors_.at(name);
    k << "|out:" << name << ':' << t.buffer()->data() << ':' << t.byte_offset();
  }
  for (std::size_t i = 0; i < selected_candidates_.size(); ++i) {
    k << "|candidate:" << state_->plan.ops()[i].candidates[selected_candidates_[i]].candidate_id;
  }
  const std::string key = k.str();
  auto entry = std::find_if(cuda->graphs.begin(), cuda->graphs.end(),
                            [&](const GraphEntry& g) { return g.key == key; });
  if (entry == cuda->graphs.end()) {
    GraphEntry fresh;
    fresh.key = key;
    CUTRITON_RETURN_IF_ERROR(drv::Check(
        api.cuStreamBeginCapture(cuda->active_stream, CU_STREAM_CAPTURE_MODE_GLOBAL), "cuStreamBeginCapture"));
    const Status captured = enqueue();
    const Status ended = drv::Check(api.cuStreamEndCapture(cuda->active_stream, &fresh.graph), "cuStreamEndCapture");
    if (!captured.ok() || !ended.ok()) {
      if (fresh.graph != nullptr) api.cuGraphDestroy(fresh.graph);
      return captured.ok() ? ended : captured;
    }
    const Status instantiated =
        drv::Check(api.cuGraphInstantiateWithFlags(&fresh.exec, fresh.graph, 0), "cuGraphInstantiate");
    if (!instantiated.ok()) {
      api.cuGraphDestroy(fresh.graph);
      return instantiated;
    }
    const std::size_t capacity = std::max<std::size_t>(1, state_->plan.cuda_graph_cache_capacity());
    if (cuda->graphs.size() >= capacity) {
      auto oldest = std::min_element(cuda->graphs.begin(), cuda->graphs.end(),
                                     [](const GraphEntry& a, const GraphEntry& b) { return a.last_used < b.last_used; });
      api.cuGraphExecDestroy(oldest->exec);
      api.cuGraphDestroy(oldest->graph);
      cuda->graphs.erase(oldest);
    }
    cuda->graphs.push_back(std::move(fresh));
    entry = std::prev(cuda->graphs.end());
  }
  entry->last_used = ++cuda->clock;
  CUTRITON_RETURN_IF_ERROR(drv::Check(api.cuGraphLaunch(entry->exec, cuda->active_stream), "cuGraphLaunch"));
  run_pending_ = true;
  return Status::OK();
}

Status ExecutionContext::Synchronize() {
  if (!run_pending_) return Status::OK();
  if (state_->plan.backend_options().device.type != DeviceType::kCUDA) {
    run_pending_ = false;
    return Status::OK();
  }
  auto* cuda = static_cast<CudaState*>(cuda_state_);
  const auto& api = drv::Get();
  run_pending_ = false;
  CUTRITON_RETURN_IF_ERROR(drv::Check(api.cuCtxSetCurrent(cuda->context), "cuCtxSetCurrent"));
  CUTRITON_RETURN_IF_ERROR(drv::Check(api.cuStreamSynchronize(cuda->active_stream), "cuStreamSynchronize"));
  if (cuda->error_host->code != 0) {
    std::ostringstream message;
    message << "a kernel abandoned a bounded wait (code " << cuda->error_host->code << ", site "
            << cuda->error_host->site << ", block " << cuda->error_host->block << ")";
    std::memset(cuda->error_host, 0, sizeof(ErrorBlock));
    return Status::RuntimeError(message.str());
  }
  profiler_.Clear();
  if (state_->plan.enable_profiling()) {
    for (std::size_t i = 0; i < state_->plan.ops().size(); ++i) {
      const PlanOp& op = state_->plan.ops()[i];
      const EventPair& events = cuda->events[i];
      float ms = 0.0f;
      if (events.timed) {
        CUTRITON_RETURN_IF_ERROR(drv::Check(api.cuEventElapsedTime(&ms, events.start, events.end), "cuEventElapsedTime"));
      }
      profiler_.Record(op.node_name, op.backend_name, static_cast<double>(ms));
    }
  }
  return Status::OK();
}

void ExecutionContext::InvalidateCudaGraph() {
  auto* cuda = static_cast<CudaState*>(cuda_state_);
  if (cuda == nullptr) return;
  drv::Get().cuCtxSetCurrent(cuda->context);
  DestroyGraphs(cuda);
}

}  // namespace cutriton
