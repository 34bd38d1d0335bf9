#pragma once

// Engine (shared compiled state) and ExecutionContext (one reusable run
// session). API of the reference's include/cutriton/runtime/engine.h:20-93.
//
// An ExecutionContext owns its stream, workspace, intermediate tensors,
// profiler and CUDA Graph cache. It is not thread-safe and admits at most one
// pending run; concurrent work uses one context per thread (one per GPU for
// batch-sharded inference).

#include <memory>
#include <string>
#include <unordered_map>
#include <vector>

#include "cutriton/backend/backend.h"
#include "cutriton/core/status.h"
#include "cutriton/runtime/executable_plan.h"
#include "cutriton/runtime/profiler.h"

namespace cutriton {

class ExecutionContext;
class EngineState;

class Engine {
 public:
  explicit Engine(ExecutablePlan plan);
  const ExecutablePlan& plan() const;
  std::unique_ptr<ExecutionContext> CreateExecutionContext() const;

 private:
  std::shared_ptr<EngineState> state_;
};

class ExecutionContext {
 public:
  explicit ExecutionContext(std::shared_ptr<EngineState> state);
  ~ExecutionContext();
  ExecutionContext(const ExecutionContext&) = delete;
  ExecutionContext& operator=(const ExecutionContext&) = delete;

  // Graph-boundary tensors must match the plan exactly (shape, dtype, layout,
  // device and byte range). Rebinding invalidates nothing already captured:
  // CUDA Graphs are keyed on the bound addresses.
  Status BindInput(const std::string& name, Tensor tensor);
  Status BindOutput(const std::string& name, Tensor tensor);
  Status SelectShapeProfile(const std::string& name);
  Status SetInputShape(const std::string& name, std::vector<int64_t> shape);
  Status ResolveShapes();
  const TensorDesc* GetResolvedTensorDesc(const std::string& name) const;
  // RunAsync(nullptr) followed by Synchronize().
  Status Run();
  // Enqueues the plan on `stream` (a CUstream on the plan's device, or
  // nullptr for the context's own stream).
  Status RunAsync(void* stream);
  // Waits for the pending run, collects profiling events and checks the
  // device-side error word of the kernels (bounded waits that expired).
  Status Synchronize();
  bool run_pending() const;

  const Profiler& profiler() const;
  std::size_t cached_cuda_graph_count() const;
  std::size_t loaded_cuda_module_count() const;
  // Every tensor the plan touches: bound inputs/outputs, device constants and
  // the workspace views of the intermediates (valid after the first run).
  const std::unordered_map<std::string, Tensor>& tensors() const;
  // Candidate index chosen for each plan op (after the first run).
  const std::vector<std::size_t>& selected_candidates() const;
  // Pins plan op `op` to candidate `candidate`, overriding the default and
  // the tuner for this context (used to test every variant; extension).
  Status SelectCandidate(std::size_t op, std::size_t candidate);

 private:
  // Lazy preparation stages of RunAsync; each rebuilds only what changed.
  Status PrepareTensors();
  Status ValidateBindings() const;
  Status PrepareTuning();
  Status PrepareKernels();
  void InvalidateCudaGraph();
  const Graph& ActiveGraph() const;
  const MemoryPlan& ActiveMemoryPlan() const;

  // All mutable per-context state (shapes, bindings, workspace, kernels,
  // device resources); defined in the runtime, so this header needs no CUDA.
  struct Session;
  std::shared_ptr<EngineState> state_;
  std::unique_ptr<Session> session_;
};

}  // namespace cutriton
