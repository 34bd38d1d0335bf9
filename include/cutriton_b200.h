/* C ABI of the sm_100a CUTriton execution backend (libcutriton_b200.so).
 *
 * The reference engine exposes a C++17 API only (include/cutriton/**); a
 * foreign caller (ctypes, cgo, JNI, N-API) binds this flat C surface instead.
 * Each entry point wraps one call of that C++ API, which this library also
 * exports unchanged (include/cutriton/cutriton.h). Plain pointers and sizes,
 * no C++ types, no exceptions. Every function returning int returns a
 * ctb_code; on failure ctb_last_error() gives the message of the calling
 * thread's last failing call.
 *
 * Threading follows the C++ API: models and engines may be shared read-only
 * after construction; one context is used by one thread at a time and has at
 * most one pending run.
 */
#ifndef CUTRITON_B200_H_
#define CUTRITON_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Mirrors cutriton::ErrorCode (include/cutriton/core/status.h:9-18 of the
 * reference). */
typedef enum {
  CTB_OK = 0,
  CTB_INVALID_ARGUMENT = 1,
  CTB_NOT_FOUND = 2,
  CTB_ALREADY_EXISTS = 3,
  CTB_UNSUPPORTED = 4,
  CTB_SHAPE_ERROR = 5,
  CTB_RUNTIME_ERROR = 6,
  CTB_INTERNAL = 7
} ctb_code;

/* Mirrors cutriton::DataType (reference include/cutriton/core/tensor.h:16-22). */
typedef enum {
  CTB_DTYPE_UNKNOWN = 0,
  CTB_DTYPE_FLOAT32 = 1,
  CTB_DTYPE_FLOAT16 = 2,
  CTB_DTYPE_INT32 = 3,
  CTB_DTYPE_INT64 = 4
} ctb_dtype;

/* Mirrors cutriton::TuningMode (reference include/cutriton/runtime/tuning.h:7-12). */
typedef enum {
  CTB_TUNING_DISABLED = 0,
  CTB_TUNING_USE_CACHE = 1,
  CTB_TUNING_TUNE_ON_MISS = 2,
  CTB_TUNING_FORCE_RETUNE = 3
} ctb_tuning_mode;

#define CTB_MAX_RANK 8

typedef struct ctb_model_s* ctb_model;
typedef struct ctb_engine_s* ctb_engine;
typedef struct ctb_context_s* ctb_context;

/* Message of the calling thread's last failing call ("" after success). */
const char* ctb_last_error(void);
/* ABI version of this header (major*100 + minor). */
int ctb_abi_version(void);

/* ---- Model / Graph: cutriton::Model, cutriton::Graph
 *      (reference include/cutriton/ir/graph.h:95-101,145) ---------------- */
int ctb_model_create(ctb_model* out);
void ctb_model_destroy(ctb_model model);
/* Graph::AddInput. A dimension <= 0 marks a dynamic axis (shape profiles). */
int ctb_graph_add_input(ctb_model model, const char* name, int dtype, int rank,
                        const int64_t* shape, const char* layout);
/* Graph::AddOutput. */
int ctb_graph_add_output(ctb_model model, const char* name);
/* Graph::AddNode. */
int ctb_graph_add_node(ctb_model model, const char* name, const char* op_type,
                       int num_inputs, const char* const* inputs,
                       int num_outputs, const char* const* outputs);
/* Node::SetAttribute on the most recently added node named `node`. */
int ctb_node_set_attr_int(ctb_model model, const char* node, const char* key, int64_t value);
int ctb_node_set_attr_float(ctb_model model, const char* node, const char* key, double value);
int ctb_node_set_attr_ints(ctb_model model, const char* node, const char* key,
                           int count, const int64_t* values);
/* Model::AddConstant: copies `nbytes` host bytes (little-endian elements). */
int ctb_model_add_constant(ctb_model model, const char* name, int dtype, int rank,
                           const int64_t* shape, const char* layout,
                           const void* host_data, size_t nbytes);

/* ---- Compile: cutriton::CompileOptions / BuildEngine
 *      (reference include/cutriton/compiler/compiler.h:20-46) ------------- */
typedef struct {
  const char* target;             /* "cuda_sm100" (alias "cuda_triton") */
  int device_id;
  int enable_cuda_graph;
  int enable_profiling;
  int enable_transformer_fusions;
  int enable_residual_fusion;
  const char* kernel_artifact_dir;   /* pack directory or pack.json */
  const char* tuning_cache_dir;      /* NULL: <pack>/tuning */
  int tuning_mode;                   /* ctb_tuning_mode */
  int tuning_warmup_iterations;
  int tuning_measurement_iterations;
  size_t cuda_graph_cache_capacity;
} ctb_compile_options;

/* Fills the C++ defaults (kernel_artifact_dir stays NULL). */
void ctb_compile_options_init(ctb_compile_options* options);
/* Adds one ShapeProfile range for `input` to the next ctb_engine_build of
 * `model` (profiles are named; ranges with the same profile name merge). */
int ctb_model_add_shape_profile(ctb_model model, const char* profile, const char* input,
                                int rank, const int64_t* min_shape,
                                const int64_t* opt_shape, const int64_t* max_shape);
int ctb_engine_build(ctb_model model, const ctb_compile_options* options, ctb_engine* out);
void ctb_engine_destroy(ctb_engine engine);

/* Plan inspection (ExecutablePlan::ops / graph). */
int ctb_engine_num_ops(ctb_engine engine);
/* op_type / node name copied into caller buffers (NUL-terminated, truncated). */
int ctb_engine_op_info(ctb_engine engine, int op, char* op_type, size_t op_type_len,
                       char* node_name, size_t node_name_len, int* num_candidates,
                       int* default_candidate);
int ctb_engine_candidate_id(ctb_engine engine, int op, int candidate, char* id, size_t id_len);
/* Description of a value of the compiled graph. */
int ctb_engine_value_desc(ctb_engine engine, const char* name, int* dtype, int* rank,
                          int64_t* shape /* CTB_MAX_RANK */);
size_t ctb_engine_workspace_bytes(ctb_engine engine);

/* ---- Execution: cutriton::ExecutionContext
 *      (reference include/cutriton/runtime/engine.h:30-65) --------------- */
int ctb_context_create(ctb_engine engine, ctb_context* out);
void ctb_context_destroy(ctb_context context);
/* BindInput/BindOutput of device memory on the plan's device. `nbytes` is
 * the usable size of the allocation at `device_ptr`. The context keeps only
 * the address: the caller keeps the memory alive until it rebinds the name or
 * destroys the context. */
int ctb_context_bind_input(ctb_context context, const char* name, void* device_ptr, size_t nbytes);
int ctb_context_bind_output(ctb_context context, const char* name, void* device_ptr, size_t nbytes);
int ctb_context_select_profile(ctb_context context, const char* profile);
int ctb_context_set_input_shape(ctb_context context, const char* name, int rank, const int64_t* shape);
int ctb_context_resolve_shapes(ctb_context context);
int ctb_context_resolved_desc(ctb_context context, const char* name, int* dtype, int* rank,
                              int64_t* shape /* CTB_MAX_RANK */);
int ctb_context_run(ctb_context context);
/* `stream` is a CUstream / cudaStream_t on the plan's device, or NULL. */
int ctb_context_run_async(ctb_context context, void* stream);
int ctb_context_synchronize(ctb_context context);
/* Profiler events of the last synchronized run: count, then per event its
 * name (written into `name`) and duration (ms). */
int ctb_context_profile_event_count(ctb_context context);
int ctb_context_profile_event(ctb_context context, int index, char* name, size_t name_len,
                              double* duration_ms);
size_t ctb_context_cached_graph_count(ctb_context context);
size_t ctb_context_loaded_module_count(ctb_context context);
/* Candidate chosen for plan op `op` by the last run (tuning included). */
int ctb_context_selected_candidate(ctb_context context, int op);
/* Pins plan op `op` to `candidate` for this context (ExecutionContext::
 * SelectCandidate; overrides the default and the tuner). */
int ctb_context_select_candidate(ctb_context context, int op, int candidate);

/* Extensions without a counterpart in the reference, whose harnesses copy
 * host buffers themselves around RunAsync.
 * End-to-end call with host buffers: copies each input from host memory to
 * the bound device buffer, runs, and copies each output back, all ordered on
 * `stream` (NULL: the context stream); returns after the copies complete.
 * Inputs/outputs must already be bound (their device buffers are reused). */
int ctb_context_run_host(ctb_context context, int num_inputs, const char* const* input_names,
                         const void* const* host_inputs, int num_outputs,
                         const char* const* output_names, void* const* host_outputs, void* stream);
/* Same copies and run, enqueued on `stream` (required), returning without
 * waiting: the run stays pending until ctb_context_synchronize. Host buffers
 * must be pinned for the copies to overlap other work and must stay valid
 * until then. Two contexts of one engine on two streams pipeline one step's
 * copies under the other's kernels. */
int ctb_context_run_host_async(ctb_context context, int num_inputs, const char* const* input_names,
                               const void* const* host_inputs, int num_outputs,
                               const char* const* output_names, void* const* host_outputs, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* CUTRITON_B200_H_ */
