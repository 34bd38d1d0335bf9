#pragma once

// Kernel Pack (pack.json schema v2) model: what a kernel binary is, how its
// parameters are bound from graph tensors/attributes, and how its launch grid
// is computed. API of the reference's include/cutriton/backend/kernel_artifact.h
// with sm_100a extensions:
//   * binary_format "cubin" (the reference accepts "ptx" only);
//   * argument source "tensor_map": the binder encodes a CUtensorMap for TMA;
//   * argument field "prepack": the argument binds a host-side transformed copy
//     of a constant input (e.g. weights pre-split into TF32 hi/lo halves);
//   * constraints "attribute_list_eq", "dim_multiple_of", "dim_le",
//     "input_is_constant";
//   * argument source "input_numel".

#include <array>
#include <cstdint>
#include <filesystem>
#include <string>
#include <unordered_map>
#include <vector>

#include "cutriton/core/status.h"

namespace cutriton {

enum class KernelArgumentSourceKind {
  kInput,
  kOutput,
  kInputDim,
  kInputDimProduct,
  kOutputDim,
  kOutputNumElements,
  kAttributeInt64,
  kAttributeFloat64,
  kLiteralInt32,
  kRuntimeReserved,
  // sm_100a extensions
  kInputNumElements,
  kTensorMap,
};

struct KernelArgumentSource {
  KernelArgumentSourceKind kind{KernelArgumentSourceKind::kRuntimeReserved};
  int index{0};
  int axis{0};
  int begin_axis{0};
  std::string attribute_name;
  std::string alternate_attribute_name;
  int attribute_index{0};
  int64_t default_int{0};
  double default_float{0.0};
  // Name of a registered constant transform (empty: bind the tensor as is).
  std::string prepack;
  // kTensorMap: which tensor (input/output index), the box extent per
  // dimension listed innermost first, and the smem swizzle in bytes
  // (0, 32, 64 or 128). merge_inner > 1 folds that many innermost tensor
  // dimensions into one (e.g. H, W -> H*W); the box then lists one extent
  // for the folded dimension. An optional map whose strides or base are not
  // 16-byte aligned, or that the driver cannot encode for this tensor, is
  // bound as all zeros instead of failing the launch (the kernel must not use
  // it then). swizzle_atom_bytes = 32 (with a 128-byte swizzle) permutes
  // 32-byte instead of 16-byte chunks within each 128-byte row, the layout
  // of MN-major TF32 tensor-core operands.
  bool map_output{false};
  std::vector<int64_t> box;
  int swizzle_bytes{0};
  int swizzle_atom_bytes{0};
  int merge_inner{1};
  bool optional{false};
};

struct KernelArgumentSpec {
  std::string name;
  std::string type;
  KernelArgumentSource source;
};

enum class KernelConstraintKind {
  kAttributeInt64Equals,
  kInputCountEquals,
  kTensorRankEquals,
  // sm_100a extensions
  kAttributeListEquals,
  kDimMultipleOf,
  kDimLessEqual,
  kInputIsConstant,
};

// A closed constraint language: packs cannot inject code, every condition is
// parsed once and evaluated by the C++ backend.
struct KernelConstraint {
  KernelConstraintKind kind{KernelConstraintKind::kInputCountEquals};
  std::string attribute_name;
  bool tensor_is_output{false};
  int tensor_index{0};
  int axis{0};
  int64_t expected{0};
  int64_t default_value{0};
  std::vector<int64_t> expected_list;
  std::vector<int64_t> default_list;
};

enum class GridExpressionKind {
  kLiteral,
  kInputDim,
  kOutputDim,
  kInputNumElements,
  kOutputNumElements,
  kVariantMeta,
  kCeilDiv,
  kMultiply,
  // sm_100a extensions: persistent kernels size their grid to the device.
  kMinimum,         ///< min of two sub-expressions
  kDeviceSmCount,   ///< multiprocessor count of the launch device
};

// Restricted launch-grid expression tree (no code from the manifest runs).
struct GridExpression {
  GridExpressionKind kind{GridExpressionKind::kLiteral};
  int64_t literal{1};
  int tensor_index{0};
  int axis{0};
  std::string meta_name;
  std::vector<GridExpression> operands;
};

struct KernelArtifact {
  std::string pack_name;
  int pack_version{0};
  std::string generator_version;
  std::string triton_version;
  int abi_schema_version{0};
  std::string kernel_id;
  std::string op_type;
  int kernel_version{0};
  std::string variant_id;
  bool is_default{false};
  std::string symbol;
  std::filesystem::path binary_path;
  std::string binary_format;
  std::string sha256;
  std::string dtype;
  std::string layout;
  int min_compute_capability{80};
  int num_warps{4};
  int num_stages{1};
  int shared_memory_bytes{0};
  std::array<GridExpression, 3> launch_grid{};
  std::unordered_map<std::string, int64_t> launch_meta;
  int grid_divisor{1};
  // sm_100a extension: the kernel waits for the preceding grid itself
  // (griddepcontrol.wait before touching activations), so it may be launched
  // with programmatic stream serialization and overlap the previous kernel's
  // tail.
  bool programmatic_launch{false};
  std::vector<KernelArgumentSpec> arguments;
  std::vector<KernelConstraint> constraints;
  std::string identity() const { return pack_name + ":" + kernel_id + ":" + variant_id; }
};

// Immutable, validated view over one or more Kernel Packs.
class ArtifactRepository {
 public:
  Status Load(const std::vector<std::string>& paths);
  const std::vector<KernelArtifact>* Find(const std::string& op_type) const;
  const std::vector<KernelArtifact>& artifacts() const { return artifacts_; }
  const std::string& repository_hash() const { return repository_hash_; }

 private:
  std::vector<KernelArtifact> artifacts_;
  std::unordered_map<std::string, std::vector<KernelArtifact>> by_op_type_;
  std::string repository_hash_;
};

// op/dtype/layout/SM filter shared by every lowering.
class KernelCatalog {
 public:
  explicit KernelCatalog(const ArtifactRepository* repository) : repository_(repository) {}
  std::vector<const KernelArtifact*> Query(const std::string& op_type,
                                           const std::string& dtype,
                                           const std::string& layout,
                                           int compute_capability) const;

 private:
  const ArtifactRepository* repository_{nullptr};
};

// Lower-case hex SHA-256 (FIPS 180-4) of a byte string; used for pack checks.
std::string Sha256Hex(const std::string& bytes);

}  // namespace cutriton
