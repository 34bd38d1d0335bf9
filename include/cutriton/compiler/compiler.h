#pragma once

// Model -> ExecutablePlan compiler (API of the reference's
// include/cutriton/compiler/compiler.h:20-46). The default target is the
// sm_100a backend; "cuda_triton" is accepted as an alias so code written for
// the reference engine compiles unchanged.

#include <memory>
#include <string>
#include <vector>

#include "cutriton/core/status.h"
#include "cutriton/ir/graph.h"
#include "cutriton/runtime/engine.h"
#include "cutriton/runtime/executable_plan.h"
#include "cutriton/runtime/shape_profile.h"
#include "cutriton/runtime/tuning.h"

namespace cutriton {

struct CompileOptions {
  std::string target{"cuda_sm100"};
  bool allow_cpu_fallback{false};
  bool enable_cuda_graph{true};
  bool enable_profiling{true};
  bool enable_transformer_fusions{true};
  // Fuse the bottleneck tail FusedConvBatchNorm -> AddRelu into one op whose
  // epilogue adds the residual (sm_100a extension; keeps an unfused candidate).
  bool enable_residual_fusion{false};
  int device_id{0};
  std::string kernel_artifact_dir;
  std::vector<std::string> kernel_artifact_paths;
  std::string tuning_cache_dir;
  TuningMode tuning_mode{TuningMode::kUseCache};
  std::vector<ShapeProfile> shape_profiles;
  std::size_t cuda_graph_cache_capacity{4};
  int tuning_warmup_iterations{5};
  int tuning_measurement_iterations{20};
};

class Compiler {
 public:
  Status Compile(const Model& model, const CompileOptions& options,
                 ExecutablePlan* plan) const;
};

Status BuildEngine(const Model& model, const CompileOptions& options,
                   std::unique_ptr<Engine>* engine);

}  // namespace cutriton
