#pragma once

// Graph passes and the default compile pipeline (API of the reference's
// include/cutriton/ir/pass.h:14-68).

#include <memory>
#include <string>
#include <vector>

#include "cutriton/core/status.h"
#include "cutriton/ir/graph.h"

namespace cutriton {

class GraphPass {
 public:
  virtual ~GraphPass() = default;
  virtual const char* name() const = 0;
  virtual Status Run(Graph* graph) const = 0;
};

class PassManager {
 public:
  void Add(std::unique_ptr<GraphPass> pass);
  Status Run(Graph* graph) const;
  const std::vector<std::string>& executed_passes() const { return executed_passes_; }

 private:
  std::vector<std::unique_ptr<GraphPass>> passes_;
  mutable std::vector<std::string> executed_passes_;
};

std::unique_ptr<GraphPass> CreateTopologicalSortPass();
std::unique_ptr<GraphPass> CreateShapeInferencePass();
std::unique_ptr<GraphPass> CreateConstantFoldingPass();
std::unique_ptr<GraphPass> CreateDeadNodeEliminationPass();
// Conv -> BatchNormalization [-> Relu]  =>  FusedConvBatchNorm[Relu].
std::unique_ptr<GraphPass> CreateConvBatchNormReluFusionPass();
// Add -> Relu  =>  AddRelu.
std::unique_ptr<GraphPass> CreateAddReluFusionPass();
// Gemm -> Gelu  =>  GemmGelu (Gemm output single-consumer, not a graph output).
std::unique_ptr<GraphPass> CreateGemmGeluFusionPass();
// Add -> LayerNormalization  =>  SkipLayerNormalization.
std::unique_ptr<GraphPass> CreateSkipLayerNormalizationFusionPass();
// MatMul -> Gemm; default Flatten axis.
std::unique_ptr<GraphPass> CreateFlattenGemmNormalizationPass();
std::unique_ptr<GraphPass> CreateStaticShapeValidationPass();
// FusedConvBatchNorm -> AddRelu  =>  FusedConvBatchNormAddRelu (residual add +
// ReLU in the convolution epilogue). sm_100a extension.
std::unique_ptr<GraphPass> CreateConvResidualFusionPass();

// The reference pipeline: topo, shape, fold, DCE, Conv+BN(+ReLU), Add+ReLU,
// [GemmGelu, SkipLayerNorm], topo, shape, MatMul/Flatten normalisation, DCE,
// validation.
PassManager CreateDefaultCompilePasses(bool enable_transformer_fusions = true);
// Same pipeline with the residual epilogue fusion inserted after Add+ReLU.
PassManager CreateCompilePasses(bool enable_transformer_fusions, bool enable_residual_fusion);

}  // namespace cutriton
