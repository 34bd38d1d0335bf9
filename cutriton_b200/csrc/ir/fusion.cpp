#include "cutriton/ir/fusion.h"

#include <mutex>

namespace cutriton {

FusionRegistry& FusionRegistry::Global() {
  static FusionRegistry registry;
  return registry;
}

Status FusionRegistry::Register(FusionAlternative alternative) {
  if (alternative.fused_op_type.empty() || alternative.candidate_id.empty() ||
      alternative.decomposed_ops.empty()) {
    return Status::InvalidArgument("fusion alternative is incomplete");
  }
  std::unique_lock<std::shared_mutex> lock(mutex_);
  auto& list = alternatives_[alternative.fused_op_type];
  for (const auto& existing : list) {
    if (existing.candidate_id == alternative.candidate_id) {
      return Status::AlreadyExists("fusion alternative already exists: " + alternative.candidate_id);
    }
  }
  list.push_back(std::move(alternative));
  return Status::OK();
}

std::vector<FusionAlternative> FusionRegistry::Find(const std::string& fused_op_type) const {
  std::shared_lock<std::shared_mutex> lock(mutex_);
  const auto it = alternatives_.find(fused_op_type);
  return it == alternatives_.end() ? std::vector<FusionAlternative>{} : it->second;
}

void FusionRegistry::ClearForTests() {
  std::unique_lock<std::shared_mutex> lock(mutex_);
  alternatives_.clear();
}

// Fused op -> the op chain it replaces. Lowering turns each entry into an
// unfused candidate built from the sub-ops' default kernels.
Status RegisterBuiltinFusionAlternatives() {
  const FusionAlternative table[] = {
      {"FusedConvBatchNormRelu", "unfused:conv_bn_relu", {"Conv", "BatchNormalization", "Relu"}},
      {"FusedConvBatchNorm", "unfused:conv_bn", {"Conv", "BatchNormalization"}},
      {"FusedConvBatchNormAddRelu", "unfused:conv_bn_add_relu",
       {"FusedConvBatchNorm", "AddRelu"}},
      {"AddRelu", "unfused:add_relu", {"Add", "Relu"}},
      {"GemmGelu", "unfused:gemm_gelu", {"Gemm", "Gelu"}},
      {"SkipLayerNormalization", "unfused:add_layer_norm", {"Add", "LayerNormalization"}},
  };
  auto& registry = FusionRegistry::Global();
  for (const auto& entry : table) {
    const Status status = registry.Register(entry);
    if (!status.ok() && status.code() != ErrorCode::kAlreadyExists) return status;
  }
  return Status::OK();
}

}  // namespace cutriton
