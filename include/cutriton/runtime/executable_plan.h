#pragma once

// Compiled, read-only snapshot handed to an Engine (API of the reference's
// include/cutriton/runtime/executable_plan.h:16-93).

#include <string>
#include <unordered_map>
#include <vector>

#include "cutriton/backend/backend.h"
#include "cutriton/ir/graph.h"
#include "cutriton/runtime/memory_planner.h"
#include "cutriton/runtime/shape_profile.h"
#include "cutriton/runtime/tuning.h"

namespace cutriton {

struct PlanOp {
  int node_id{-1};
  std::string node_name;
  std::string op_type;
  std::string backend_name;
  std::vector<std::string> inputs;
  std::vector<std::string> outputs;
  std::vector<ExecutionCandidate> candidates;
  std::size_t selected_candidate{0};
};

struct ProfilePlan {
  ShapeProfile profile;
  Graph min_graph;
  Graph opt_graph;
  Graph max_graph;
  MemoryPlan max_memory_plan;
};

class ExecutablePlan {
 public:
  const Graph& graph() const { return graph_; }
  Graph& mutable_graph() { return graph_; }
  const std::vector<PlanOp>& ops() const { return ops_; }
  std::vector<PlanOp>& mutable_ops() { return ops_; }
  const MemoryPlan& memory_plan() const { return memory_plan_; }
  MemoryPlan& mutable_memory_plan() { return memory_plan_; }
  const std::string& target() const { return target_; }
  void set_target(std::string target) { target_ = std::move(target); }
  const BackendOptions& backend_options() const { return backend_options_; }
  BackendOptions& mutable_backend_options() { return backend_options_; }
  const std::unordered_map<std::string, Tensor>& constants() const { return constants_; }
  std::unordered_map<std::string, Tensor>& mutable_constants() { return constants_; }
  bool enable_cuda_graph() const { return enable_cuda_graph_; }
  void set_enable_cuda_graph(bool value) { enable_cuda_graph_ = value; }
  bool enable_profiling() const { return enable_profiling_; }
  void set_enable_profiling(bool value) { enable_profiling_ = value; }
  const TuningConfig& tuning_config() const { return tuning_config_; }
  TuningConfig& mutable_tuning_config() { return tuning_config_; }
  std::size_t cuda_graph_cache_capacity() const { return cuda_graph_cache_capacity_; }
  void set_cuda_graph_cache_capacity(std::size_t value) { cuda_graph_cache_capacity_ = value; }
  const std::vector<ProfilePlan>& profile_plans() const { return profile_plans_; }
  std::vector<ProfilePlan>& mutable_profile_plans() { return profile_plans_; }

 private:
  Graph graph_;
  std::vector<PlanOp> ops_;
  MemoryPlan memory_plan_;
  std::string target_;
  BackendOptions backend_options_;
  std::unordered_map<std::string, Tensor> constants_;
  bool enable_cuda_graph_{false};
  bool enable_profiling_{false};
  TuningConfig tuning_config_;
  std::size_t cuda_graph_cache_capacity_{4};
  std::vector<ProfilePlan> profile_plans_;
};

}  // namespace cutriton
