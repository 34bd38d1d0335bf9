// C ABI over the C++ API (include/cutriton_b200.h).

#include "cutriton_b200.h"

#include <cstring>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "cuda_driver.h"
#include "cutriton/cutriton.h"

using namespace cutriton;

struct ctb_model_s {
  Model model;
  std::map<std::string, ShapeProfile> profiles;
  std::vector<std::string> profile_order;
};

struct ctb_engine_s {
  std::unique_ptr<Engine> engine;
};

struct ctb_context_s {
  std::unique_ptr<ExecutionContext> context;
  int device_id{0};
  // Graph input/output descriptions of the static plan (the context may
  // outlive its engine, so they are copied).
  std::map<std::string, TensorDesc> plan_descs;
};

namespace {

thread_local std::string g_last_error;

int Report(const Status& status) {
  if (status.ok()) {
    g_last_error.clear();
    return CTB_OK;
  }
  g_last_error = status.ToString();
  return static_cast<int>(status.code());
}

int Invalid(const char* message) { return Report(Status::InvalidArgument(message)); }

DataType ToDataType(int dtype) {
  switch (dtype) {
    case CTB_DTYPE_FLOAT32: return DataType::kFloat32;
    case CTB_DTYPE_FLOAT16: return DataType::kFloat16;
    case CTB_DTYPE_INT32: return DataType::kInt32;
    case CTB_DTYPE_INT64: return DataType::kInt64;
    default: return DataType::kUnknown;
  }
}

int FromDataType(DataType dtype) {
  switch (dtype) {
    case DataType::kFloat32: return CTB_DTYPE_FLOAT32;
    case DataType::kFloat16: return CTB_DTYPE_FLOAT16;
    case DataType::kInt32: return CTB_DTYPE_INT32;
    case DataType::kInt64: return CTB_DTYPE_INT64;
    default: return CTB_DTYPE_UNKNOWN;
  }
}

bool ShapeFrom(int rank, const int64_t* dims, std::vector<int64_t>* shape) {
  if (rank < 0 || rank > CTB_MAX_RANK || (rank > 0 && dims == nullptr)) return false;
  shape->assign(dims, dims + rank);
  return true;
}

void CopyString(const std::string& text, char* out, std::size_t len) {
  if (out == nullptr || len == 0) return;
  const std::size_t n = std::min(text.size(), len - 1);
  std::memcpy(out, text.data(), n);
  out[n] = '\0';
}

void DescOut(const TensorDesc& desc, int* dtype, int* rank, int64_t* shape) {
  if (dtype != nullptr) *dtype = FromDataType(desc.dtype);
  if (rank != nullptr) *rank = static_cast<int>(desc.shape.size());
  if (shape != nullptr) {
    for (std::size_t i = 0; i < desc.shape.size() && i < CTB_MAX_RANK; ++i) shape[i] = desc.shape[i];
  }
}

Node* FindNode(ctb_model model, const char* name) {
  auto& nodes = model->model.graph().mutable_nodes();
  for (auto it = nodes.rbegin(); it != nodes.rend(); ++it) {
    if (it->name() == name) return &*it;
  }
  return nullptr;
}

const TensorDesc* BindingDesc(ctb_context c, const std::string& name) {
  if (const TensorDesc* resolved = c->context->GetResolvedTensorDesc(name)) return resolved;
  const auto it = c->plan_descs.find(name);
  return it == c->plan_descs.end() ? nullptr : &it->second;
}

}  // namespace

extern "C" {

const char* ctb_last_error(void) { return g_last_error.c_str(); }
int ctb_abi_version(void) { return 100; }

int ctb_model_create(ctb_model* out) {
  if (out == nullptr) return Invalid("model output pointer is null");
  *out = new ctb_model_s();
  return Report(Status::OK());
}

void ctb_model_destroy(ctb_model model) { delete model; }

int ctb_graph_add_input(ctb_model model, const char* name, int dtype, int rank, const int64_t* shape,
                        const char* layout) {
  if (model == nullptr || name == nullptr) return Invalid("model and name are required");
  std::vector<int64_t> dims;
  if (!ShapeFrom(rank, shape, &dims)) return Invalid("invalid rank or shape");
  TensorDesc desc(std::move(dims), ToDataType(dtype), DeviceType::kCPU, 0, layout ? layout : "NCHW");
  return Report(model->model.graph().AddInput(name, std::move(desc)));
}

int ctb_graph_add_output(ctb_model model, const char* name) {
  if (model == nullptr || name == nullptr) return Invalid("model and name are required");
  return Report(model->model.graph().AddOutput(name));
}

int ctb_graph_add_node(ctb_model model, const char* name, const char* op_type, int num_inputs,
                       const char* const* inputs, int num_outputs, const char* const* outputs) {
  if (model == nullptr || name == nullptr || op_type == nullptr || num_inputs < 0 || num_outputs < 0 ||
      (num_inputs > 0 && inputs == nullptr) || (num_outputs > 0 && outputs == nullptr)) {
    return Invalid("invalid node arguments");
  }
  std::vector<std::string> in(inputs, inputs + num_inputs);
  std::vector<std::string> out(outputs, outputs + num_outputs);
  return Report(model->model.graph().AddNode(Node(name, op_type, std::move(in), std::move(out))));
}

int ctb_node_set_attr_int(ctb_model model, const char* node, const char* key, int64_t value) {
  if (model == nullptr || node == nullptr || key == nullptr) return Invalid("invalid attribute arguments");
  Node* n = FindNode(model, node);
  if (n == nullptr) return Report(Status::NotFound(std::string("node not found: ") + node));
  n->SetAttribute(key, value);
  return Report(Status::OK());
}

int ctb_node_set_attr_float(ctb_model model, const char* node, const char* key, double value) {
  if (model == nullptr || node == nullptr || key == nullptr) return Invalid("invalid attribute arguments");
  Node* n = FindNode(model, node);
  if (n == nullptr) return Report(Status::NotFound(std::string("node not found: ") + node));
  n->SetAttribute(key, value);
  return Report(Status::OK());
}

int ctb_node_set_attr_ints(ctb_model model, const char* node, const char* key, int count, const int64_t* values) {
  if (model == nullptr || node == nullptr || key == nullptr || count < 0 || (count > 0 && values == nullptr)) {
    return Invalid("invalid attribute arguments");
  }
  Node* n = FindNode(model, node);
  if (n == nullptr) return Report(Status::NotFound(std::string("node not found: ") + node));
  n->SetAttribute(key, std::vector<int64_t>(values, values + count));
  return Report(Status::OK());
}

int ctb_model_add_constant(ctb_model model, const char* name, int dtype, int rank, const int64_t* shape,
                           const char* layout, const void* host_data, size_t nbytes) {
  if (model == nullptr || name == nullptr || (nbytes > 0 && host_data == nullptr)) {
    return Invalid("invalid constant arguments");
  }
  std::vector<int64_t> dims;
  if (!ShapeFrom(rank, shape, &dims)) return Invalid("invalid rank or shape");
  TensorDesc desc(std::move(dims), ToDataType(dtype), DeviceType::kCPU, 0, layout ? layout : "NCHW");
  if (desc.ByteSize() != nbytes) return Invalid("constant byte count does not match its shape");
  auto buffer = Buffer::AllocateHost(nbytes);
  const Status copied = buffer->CopyFromHost(host_data, nbytes);
  if (!copied.ok()) return Report(copied);
  return Report(model->model.AddConstant(name, Tensor(std::move(desc), std::move(buffer))));
}

void ctb_compile_options_init(ctb_compile_options* o) {
  if (o == nullptr) return;
  const CompileOptions d;
  o->target = "cuda_sm100";
  o->device_id = d.device_id;
  o->enable_cuda_graph = d.enable_cuda_graph ? 1 : 0;
  o->enable_profiling = d.enable_profiling ? 1 : 0;
  o->enable_transformer_fusions = d.enable_transformer_fusions ? 1 : 0;
  o->enable_residual_fusion = d.enable_residual_fusion ? 1 : 0;
  o->kernel_artifact_dir = nullptr;
  o->tuning_cache_dir = nullptr;
  o->tuning_mode = static_cast<int>(d.tuning_mode);
  o->tuning_warmup_iterations = d.tuning_warmup_iterations;
  o->tuning_measurement_iterations = d.tuning_measurement_iterations;
  o->cuda_graph_cache_capacity = d.cuda_graph_cache_capacity;
}

int ctb_model_add_shape_profile(ctb_model model, const char* profile, const char* input, int rank,
                                const int64_t* min_shape, const int64_t* opt_shape, const int64_t* max_shape) {
  if (model == nullptr || profile == nullptr || input == nullptr) return Invalid("invalid profile arguments");
  ShapeRange range;
  if (!ShapeFrom(rank, min_shape, &range.min) || !ShapeFrom(rank, opt_shape, &range.opt) ||
      !ShapeFrom(rank, max_shape, &range.max)) {
    return Invalid("invalid profile shapes");
  }
  auto found = model->profiles.find(profile);
  if (found == model->profiles.end()) {
    model->profile_order.push_back(profile);
    found = model->profiles.emplace(profile, ShapeProfile{profile, {}}).first;
  }
  found->second.inputs[input] = std::move(range);
  return Report(Status::OK());
}

int ctb_engine_build(ctb_model model, const ctb_compile_options* o, ctb_engine* out) {
  if (model == nullptr || o == nullptr || out == nullptr) return Invalid("invalid build arguments");
  CompileOptions options;
  if (o->target != nullptr) options.target = o->target;
  options.device_id = o->device_id;
  options.enable_cuda_graph = o->enable_cuda_graph != 0;
  options.enable_profiling = o->enable_profiling != 0;
  options.enable_transformer_fusions = o->enable_transformer_fusions != 0;
  options.enable_residual_fusion = o->enable_residual_fusion != 0;
  if (o->kernel_artifact_dir != nullptr) options.kernel_artifact_paths = {o->kernel_artifact_dir};
  if (o->tuning_cache_dir != nullptr) options.tuning_cache_dir = o->tuning_cache_dir;
  if (o->tuning_mode < CTB_TUNING_DISABLED || o->tuning_mode > CTB_TUNING_FORCE_RETUNE) {
    return Invalid("invalid tuning mode");
  }
  options.tuning_mode = static_cast<TuningMode>(o->tuning_mode);
  options.tuning_warmup_iterations = o->tuning_warmup_iterations;
  options.tuning_measurement_iterations = o->tuning_measurement_iterations;
  options.cuda_graph_cache_capacity = o->cuda_graph_cache_capacity;
  for (const auto& name : model->profile_order) options.shape_profiles.push_back(model->profiles.at(name));
  auto holder = std::make_unique<ctb_engine_s>();
  const Status built = BuildEngine(model->model, options, &holder->engine);
  if (!built.ok()) return Report(built);
  *out = holder.release();
  return Report(Status::OK());
}

void ctb_engine_destroy(ctb_engine engine) { delete engine; }

int ctb_engine_num_ops(ctb_engine engine) {
  return engine == nullptr ? -1 : static_cast<int>(engine->engine->plan().ops().size());
}

int ctb_engine_op_info(ctb_engine engine, int op, char* op_type, size_t op_type_len, char* node_name,
                       size_t node_name_len, int* num_candidates, int* default_candidate) {
  if (engine == nullptr) return Invalid("engine is null");
  const auto& ops = engine->engine->plan().ops();
  if (op < 0 || static_cast<std::size_t>(op) >= ops.size()) return Invalid("op index out of range");
  const PlanOp& p = ops[static_cast<std::size_t>(op)];
  CopyString(p.op_type, op_type, op_type_len);
  CopyString(p.node_name, node_name, node_name_len);
  if (num_candidates != nullptr) *num_candidates = static_cast<int>(p.candidates.size());
  if (default_candidate != nullptr) *default_candidate = static_cast<int>(p.selected_candidate);
  return Report(Status::OK());
}

int ctb_engine_candidate_id(ctb_engine engine, int op, int candidate, char* id, size_t id_len) {
  if (engine == nullptr) return Invalid("engine is null");
  const auto& ops = engine->engine->plan().ops();
  if (op < 0 || static_cast<std::size_t>(op) >= ops.size()) return Invalid("op index out of range");
  const auto& candidates = ops[static_cast<std::size_t>(op)].candidates;
  if (candidate < 0 || static_cast<std::size_t>(candidate) >= candidates.size()) return Invalid("candidate out of range");
  CopyString(candidates[static_cast<std::size_t>(candidate)].candidate_id, id, id_len);
  return Report(Status::OK());
}

int ctb_engine_value_desc(ctb_engine engine, const char* name, int* dtype, int* rank, int64_t* shape) {
  if (engine == nullptr || name == nullptr) return Invalid("invalid arguments");
  const ValueDesc* v = engine->engine->plan().graph().FindValue(name);
  if (v == nullptr) return Report(Status::NotFound(std::string("value not found: ") + name));
  DescOut(v->tensor, dtype, rank, shape);
  return Report(Status::OK());
}

size_t ctb_engine_workspace_bytes(ctb_engine engine) {
  return engine == nullptr ? 0 : engine->engine->plan().memory_plan().workspace_size_bytes;
}

int ctb_context_create(ctb_engine engine, ctb_context* out) {
  if (engine == nullptr || out == nullptr) return Invalid("invalid context arguments");
  auto holder = std::make_unique<ctb_context_s>();
  holder->context = engine->engine->CreateExecutionContext();
  const ExecutablePlan& plan = engine->engine->plan();
  holder->device_id = plan.backend_options().device.id;
  for (const auto* names : {&plan.graph().inputs(), &plan.graph().outputs()}) {
    for (const auto& name : *names) {
      if (const ValueDesc* v = plan.graph().FindValue(name)) holder->plan_descs[name] = v->tensor;
    }
  }
  *out = holder.release();
  return Report(Status::OK());
}

void ctb_context_destroy(ctb_context context) { delete context; }

static int Bind(ctb_context c, const char* name, void* ptr, size_t nbytes, bool input) {
  if (c == nullptr || name == nullptr || ptr == nullptr) return Invalid("invalid binding arguments");
  const TensorDesc* desc = BindingDesc(c, name);
  if (desc == nullptr) return Report(Status::NotFound("not a graph input/output: " + std::string(name)));
  const TensorDesc expected = *desc;
  auto buffer = Buffer::WrapExternal(ptr, nbytes, expected.device_type, expected.device_id);
  Tensor tensor(expected, std::move(buffer));
  return Report(input ? c->context->BindInput(name, std::move(tensor)) : c->context->BindOutput(name, std::move(tensor)));
}

int ctb_context_bind_input(ctb_context c, const char* name, void* ptr, size_t nbytes) {
  return Bind(c, name, ptr, nbytes, true);
}

int ctb_context_bind_output(ctb_context c, const char* name, void* ptr, size_t nbytes) {
  return Bind(c, name, ptr, nbytes, false);
}

int ctb_context_select_profile(ctb_context c, const char* profile) {
  if (c == nullptr || profile == nullptr) return Invalid("invalid arguments");
  return Report(c->context->SelectShapeProfile(profile));
}

int ctb_context_set_input_shape(ctb_context c, const char* name, int rank, const int64_t* shape) {
  if (c == nullptr || name == nullptr) return Invalid("invalid arguments");
  std::vector<int64_t> dims;
  if (!ShapeFrom(rank, shape, &dims)) return Invalid("invalid rank or shape");
  return Report(c->context->SetInputShape(name, std::move(dims)));
}

int ctb_context_resolve_shapes(ctb_context c) {
  if (c == nullptr) return Invalid("context is null");
  return Report(c->context->ResolveShapes());
}

int ctb_context_resolved_desc(ctb_context c, const char* name, int* dtype, int* rank, int64_t* shape) {
  if (c == nullptr || name == nullptr) return Invalid("invalid arguments");
  const TensorDesc* desc = BindingDesc(c, name);
  if (desc == nullptr) return Report(Status::NotFound(std::string("no resolved description for ") + name));
  DescOut(*desc, dtype, rank, shape);
  return Report(Status::OK());
}

int ctb_context_run(ctb_context c) {
  if (c == nullptr) return Invalid("context is null");
  return Report(c->context->Run());
}

int ctb_context_run_async(ctb_context c, void* stream) {
  if (c == nullptr) return Invalid("context is null");
  return Report(c->context->RunAsync(stream));
}

int ctb_context_synchronize(ctb_context c) {
  if (c == nullptr) return Invalid("context is null");
  return Report(c->context->Synchronize());
}

int ctb_context_profile_event_count(ctb_context c) {
  return c == nullptr ? -1 : static_cast<int>(c->context->profiler().events().size());
}

int ctb_context_profile_event(ctb_context c, int index, char* name, size_t name_len, double* duration_ms) {
  if (c == nullptr) return Invalid("context is null");
  const auto& events = c->context->profiler().events();
  if (index < 0 || static_cast<std::size_t>(index) >= events.size()) return Invalid("event index out of range");
  CopyString(events[static_cast<std::size_t>(index)].name, name, name_len);
  if (duration_ms != nullptr) *duration_ms = events[static_cast<std::size_t>(index)].duration_ms;
  return Report(Status::OK());
}

size_t ctb_context_cached_graph_count(ctb_context c) { return c == nullptr ? 0 : c->context->cached_cuda_graph_count(); }
size_t ctb_context_loaded_module_count(ctb_context c) { return c == nullptr ? 0 : c->context->loaded_cuda_module_count(); }

int ctb_context_selected_candidate(ctb_context c, int op) {
  if (c == nullptr) return -1;
  const auto& selected = c->context->selected_candidates();
  if (op < 0 || static_cast<std::size_t>(op) >= selected.size()) return -1;
  return static_cast<int>(selected[static_cast<std::size_t>(op)]);
}

int ctb_context_select_candidate(ctb_context c, int op, int candidate) {
  if (c == nullptr || op < 0 || candidate < 0) return Invalid("invalid arguments");
  return Report(c->context->SelectCandidate(static_cast<std::size_t>(op), static_cast<std::size_t>(candidate)));
}

namespace {

// H2D copies of the inputs, the run, D2H copies of the outputs. With a stream
// everything is enqueued on it and the run stays pending (the caller
// synchronizes); without one the copies are synchronous around a synchronous
// run on the context stream.
int EnqueueRunHost(ctb_context c, int num_inputs, const char* const* input_names, const void* const* host_inputs,
                   int num_outputs, const char* const* output_names, void* const* host_outputs, void* stream,
                   bool wait) {
  if (c == nullptr || num_inputs < 0 || num_outputs < 0) return Invalid("invalid arguments");
  if (c->context->run_pending()) return Report(Status::RuntimeError("a run is already pending"));
  Status status = drv::Ensure();
  if (!status.ok()) return Report(status);
  const auto& api = drv::Get();
  CUdevice device{};
  CUcontext cu_context{};
  status = drv::RetainPrimaryContext(c->device_id, &device, &cu_context);
  if (!status.ok()) return Report(status);
  struct Release {
    CUdevice d;
    ~Release() { drv::Get().cuDevicePrimaryCtxRelease(d); }
  } release{device};
  const auto& tensors = c->context->tensors();
  auto device_of = [&](const char* name, CUdeviceptr* ptr, std::size_t* bytes) -> Status {
    const auto it = tensors.find(name);
    if (it == tensors.end() || !it->second.defined()) {
      return Status::InvalidArgument(std::string("tensor is not bound: ") + name);
    }
    *ptr = static_cast<CUdeviceptr>(reinterpret_cast<std::uintptr_t>(it->second.buffer()->data())) +
           it->second.byte_offset();
    *bytes = it->second.desc().ByteSize();
    return Status::OK();
  };
  const CUstream s = reinterpret_cast<CUstream>(stream);
  for (int i = 0; i < num_inputs; ++i) {
    CUdeviceptr ptr{};
    std::size_t bytes = 0;
    status = device_of(input_names[i], &ptr, &bytes);
    if (!status.ok()) return Report(status);
    status = s != nullptr ? drv::Check(api.cuMemcpyHtoDAsync(ptr, host_inputs[i], bytes, s), "cuMemcpyHtoDAsync")
                          : drv::Check(api.cuMemcpyHtoD(ptr, host_inputs[i], bytes), "cuMemcpyHtoD");
    if (!status.ok()) return Report(status);
  }
  if (s == nullptr) {
    status = c->context->Run();
    if (!status.ok()) return Report(status);
  } else {
    status = c->context->RunAsync(stream);
    if (!status.ok()) return Report(status);
  }
  for (int i = 0; i < num_outputs; ++i) {
    CUdeviceptr ptr{};
    std::size_t bytes = 0;
    status = device_of(output_names[i], &ptr, &bytes);
    if (status.ok()) {
      status = s != nullptr ? drv::Check(api.cuMemcpyDtoHAsync(host_outputs[i], ptr, bytes, s), "cuMemcpyDtoHAsync")
                            : drv::Check(api.cuMemcpyDtoH(host_outputs[i], ptr, bytes), "cuMemcpyDtoH");
    }
    if (!status.ok()) {
      if (s != nullptr) (void)c->context->Synchronize();
      return Report(status);
    }
  }
  return Report(s != nullptr && wait ? c->context->Synchronize() : Status::OK());
}

}  // namespace

int ctb_context_run_host(ctb_context c, int num_inputs, const char* const* input_names,
                         const void* const* host_inputs, int num_outputs, const char* const* output_names,
                         void* const* host_outputs, void* stream) {
  return EnqueueRunHost(c, num_inputs, input_names, host_inputs, num_outputs, output_names, host_outputs, stream,
                        true);
}

int ctb_context_run_host_async(ctb_context c, int num_inputs, const char* const* input_names,
                               const void* const* host_inputs, int num_outputs, const char* const* output_names,
                               void* const* host_outputs, void* stream) {
  if (stream == nullptr) return Invalid("ctb_context_run_host_async needs a stream");
  return EnqueueRunHost(c, num_inputs, input_names, host_inputs, num_outputs, output_names, host_outputs, stream,
                        false);
}

}  // extern "C"
