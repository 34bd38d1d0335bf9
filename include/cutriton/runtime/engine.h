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
  bool run_pending() const { return run_pending_; }

  const Profiler& profiler() const { return profiler_; }
  std::size_t cached_cuda_graph_count() const;
  std::size_t loaded_cuda_module_count() const;
  const std::unordered_map<std::string, Tensor>& tensors() const { return tensors_; }
  // Candidate index chosen for each plan op (after the first run).
  const std::vector<std::size_t>& selected_candidates() const { return selected_candidates_; }
  // Pins plan op `op` to candidate `candidate`, overriding the default and
  // the tuner for this context (used to test every variant; extension).
  Status SelectCandidate(std::size_t op, std::size_t candidate);

 private:
  Status PrepareKernels();
  Status PrepareTuning();
  Status PrepareTensors();
  Status ValidateBindings() const;
  void InvalidateCudaGraph();
  const Graph& ActiveGraph() const;
  const MemoryPlan& ActiveMemoryPlan() const;

  std::shared_ptr<EngineState> state_;
  bool kernels_prepared_{false};
  bool tensors_prepared_{false};
  bool run_pending_{false};
  bool tuning_prepared_{false};
  std::vector<std::size_t> selected_candidates_;
  std::unordered_map<std::size_t, std::size_t> pinned_candidates_;
  int selected_profile_{-1};
  std::unordered_map<std::string, std::vector<int64_t>> input_shapes_;
  Graph resolved_graph_;
  bool shapes_resolved_{false};
  std::vector<std::vector<std::unique_ptr<OpKernel>>> kernels_;
  std::unordered_map<std::string, Tensor> tensors_;
  std::shared_ptr<Buffer> workspace_;
  Profiler profiler_;
  void* cuda_state_{nullptr};
};

}  // namespace cutriton
