// Generic manifest-driven launcher: module cache, argument binder, grid
// evaluator and one cuLaunchKernel per compute step.
//
// Behaviour follows the reference launcher (src/backend/cuda_launcher.cpp:
// CudaModuleCache 47-118, ArgumentBinder::Bind 129-199, EvaluateGridExpression
// 291-377, InvocationKernel::Compute 394-423). sm_100a additions:
//   * cubin modules (cuModuleLoadData takes cubin and PTX alike);
//   * the dynamic shared-memory opt-in for kernels above 48 KB, set once per
//     function when it is first resolved;
//   * "tensor_map" parameters: a CUtensorMap (128 B, 64-B aligned) encoded
//     with cuTensorMapEncodeTiled over the bound tensor;
//   * "prepack" parameters bind the derived constant "<name>::<prepack>";
//   * the first runtime_reserved parameter carries the context's error block.

#include <array>
#include <cstdint>
#include <cstring>
#include <fstream>
#include <limits>
#include <mutex>
#include <sstream>
#include <unordered_map>

#include "../cuda_driver.h"
#include "cutriton/backend/backend.h"
#include "cutriton/core/buffer.h"
#include "prepack.h"

namespace cutriton {

class CudaModuleCache {
 public:
  explicit CudaModuleCache(int device_id) : device_id_(device_id) {}
  ~CudaModuleCache() {
    if (context_ == nullptr) return;
    std::lock_guard<std::mutex> lock(mutex_);
    const auto& api = drv::Get();
    api.cuCtxSetCurrent(context_);
    for (const auto& entry : modules_) api.cuModuleUnload(entry.second);
    api.cuDevicePrimaryCtxRelease(device_);
  }

  Status Initialize() { return drv::RetainPrimaryContext(device_id_, &device_, &context_); }

  // Resolves (loading on first use) the kernel function of an artifact.
  Status GetFunction(const KernelArtifact& artifact, CUfunction* function) {
    if (function == nullptr) return Status::InvalidArgument("CUfunction output is null");
    std::lock_guard<std::mutex> lock(mutex_);
    const auto& api = drv::Get();
    CUTRITON_RETURN_IF_ERROR(drv::Check(api.cuCtxSetCurrent(context_), "cuCtxSetCurrent"));
    auto module = modules_.find(artifact.sha256);
    if (module == modules_.end()) {
      std::ifstream in(artifact.binary_path, std::ios::binary);
      if (!in) return Status::NotFound("kernel binary not found: " + artifact.binary_path.string());
      std::ostringstream bytes;
      bytes << in.rdbuf();
      std::string image = bytes.str();
      image.push_back('\0');  // PTX images must be NUL-terminated; harmless for cubin
      CUmodule loaded{};
      CUTRITON_RETURN_IF_ERROR(drv::Check(api.cuModuleLoadData(&loaded, image.data()), "cuModuleLoadData"));
      module = modules_.emplace(artifact.sha256, loaded).first;
    }
    const std::string key = artifact.sha256 + ":" + artifact.symbol;
    const auto cached = functions_.find(key);
    if (cached != functions_.end()) {
      *function = cached->second;
      return Status::OK();
    }
    CUfunction resolved{};
    CUTRITON_RETURN_IF_ERROR(drv::Check(
        api.cuModuleGetFunction(&resolved, module->second, artifact.symbol.c_str()),
        "cuModuleGetFunction"));
    if (artifact.shared_memory_bytes > 48 * 1024) {
      CUTRITON_RETURN_IF_ERROR(drv::Check(
          api.cuFuncSetAttribute(resolved, CU_FUNC_ATTRIBUTE_MAX_DYNAMIC_SHARED_SIZE_BYTES,
                                 artifact.shared_memory_bytes),
          "cuFuncSetAttribute(MAX_DYNAMIC_SHARED_SIZE_BYTES)"));
    }
    functions_.emplace(key, resolved);
    *function = resolved;
    return Status::OK();
  }

  std::size_t size() const {
    std::lock_guard<std::mutex> lock(mutex_);
    return modules_.size();
  }

 private:
  int device_id_{0};
  mutable std::mutex mutex_;
  CUdevice device_{};
  CUcontext context_{nullptr};
  std::unordered_map<std::string, CUmodule> modules_;
  std::unordered_map<std::string, CUfunction> functions_;
};

namespace {

const Tensor* FindTensor(KernelContext* context, const std::string& name) {
  const auto it = context->tensors->find(name);
  return (it == context->tensors->end() || !it->second.defined()) ? nullptr : &it->second;
}

CUdeviceptr DeviceAddress(const Tensor& tensor) {
  return static_cast<CUdeviceptr>(reinterpret_cast<std::uintptr_t>(tensor.buffer()->data())) +
         tensor.byte_offset();
}

Status TensorAt(const std::vector<std::string>& names, int index, const std::string& prepack,
                KernelContext* context, const Tensor** tensor) {
  if (index < 0 || static_cast<std::size_t>(index) >= names.size()) {
    return Status::InvalidArgument("kernel tensor argument index is invalid");
  }
  const std::string& base = names[static_cast<std::size_t>(index)];
  const std::string name = prepack.empty() ? base : PrepackedName(base, prepack);
  *tensor = FindTensor(context, name);
  return *tensor == nullptr ? Status::NotFound("kernel tensor argument is not bound: " + name)
                            : Status::OK();
}

Status Int32From(int64_t value, const char* what, int32_t* out) {
  if (value <= 0 || value > std::numeric_limits<int32_t>::max()) {
    return Status::ShapeError(std::string("kernel ") + what + " is out of the int32 range");
  }
  *out = static_cast<int32_t>(value);
  return Status::OK();
}

int64_t AttributeInt(const Node& node, const KernelArgumentSource& s) {
  if (const auto list = node.GetAttribute<std::vector<int64_t>>(s.attribute_name)) {
    if (s.attribute_index >= 0 && static_cast<std::size_t>(s.attribute_index) < list->size()) {
      return (*list)[static_cast<std::size_t>(s.attribute_index)];
    }
  }
  if (const auto scalar = node.GetAttribute<int64_t>(s.attribute_name)) return *scalar;
  return s.default_int;
}

double AttributeFloat(const Node& node, const KernelArgumentSource& s) {
  if (const auto primary = node.GetAttribute<double>(s.attribute_name)) return *primary;
  if (!s.alternate_attribute_name.empty()) {
    if (const auto alternate = node.GetAttribute<double>(s.alternate_attribute_name)) return *alternate;
  }
  return s.default_float;
}

Status EncodeTensorMap(const Tensor& tensor, const KernelArgumentSource& s, CUtensorMap* map) {
  const TensorDesc& desc = tensor.desc();
  const std::size_t tensor_rank = desc.shape.size();
  const std::size_t merge = static_cast<std::size_t>(s.merge_inner);
  if (merge > tensor_rank || tensor_rank - merge + 1 != s.box.size()) {
    if (s.optional) {  // a map that does not fit this tensor's rank is bound as zeros
      std::memset(map, 0, sizeof(*map));
      return Status::OK();
    }
    return Status::ShapeError("tensor_map box rank differs from the tensor rank");
  }
  const std::size_t rank = tensor_rank - merge + 1;
  CUtensorMapDataType type;
  switch (desc.dtype) {
    case DataType::kFloat32: type = CU_TENSOR_MAP_DATA_TYPE_FLOAT32; break;
    case DataType::kFloat16: type = CU_TENSOR_MAP_DATA_TYPE_FLOAT16; break;
    default: return Status::Unsupported("tensor_map supports float32/float16 tensors");
  }
  const std::size_t element = ElementSize(desc.dtype);
  cuuint64_t dims[5];
  cuuint64_t strides[4];
  cuuint32_t box[5];
  cuuint32_t element_strides[5];
  // Innermost (folded) dimension first.
  int64_t inner = 1;
  for (std::size_t i = 0; i < merge; ++i) inner *= desc.shape[tensor_rank - 1 - i];
  std::uint64_t running = element;
  bool aligned = true;
  for (std::size_t i = 0; i < rank; ++i) {
    const int64_t extent = i == 0 ? inner : desc.shape[rank - 1 - i];
    dims[i] = static_cast<cuuint64_t>(extent);
    box[i] = static_cast<cuuint32_t>(s.box[i]);
    element_strides[i] = 1;
    if (i > 0) {
      strides[i - 1] = running;
      aligned = aligned && running % 16 == 0;
    }
    running *= static_cast<std::uint64_t>(extent);
  }
  void* address = reinterpret_cast<void*>(DeviceAddress(tensor));
  aligned = aligned && reinterpret_cast<std::uintptr_t>(address) % 16 == 0;
  if (s.optional && !aligned) {
    std::memset(map, 0, sizeof(*map));
    return Status::OK();
  }
  CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_NONE;
  if (s.swizzle_bytes == 32) swizzle = CU_TENSOR_MAP_SWIZZLE_32B;
  if (s.swizzle_bytes == 64) swizzle = CU_TENSOR_MAP_SWIZZLE_64B;
  if (s.swizzle_bytes == 128) {
    swizzle = s.swizzle_atom_bytes == 32 ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B;
  }
  const CUresult result = drv::Get().cuTensorMapEncodeTiled(
      map, type, static_cast<cuuint32_t>(rank), address, dims, strides, box, element_strides,
      CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (result != CUDA_SUCCESS && s.optional) {
    // An optional map that does not fit this tensor is bound as zeros; the
    // kernel checks the same conditions before using it.
    std::memset(map, 0, sizeof(*map));
    return Status::OK();
  }
  return drv::Check(result, "cuTensorMapEncodeTiled");
}

// Parameter storage for one launch. Pointers into it stay valid until the
// next Bind on the same object (capacity is reserved up front).
struct BoundParameters {
  union Scalar {
    CUdeviceptr pointer;
    int32_t i32;
    float f32;
  };
  std::vector<Scalar> scalars;
  std::vector<CUtensorMap> maps;
  std::vector<void*> pointers;
};

Status BindArguments(const KernelInvocation& inv, KernelContext* context, BoundParameters* out) {
  const auto& args = inv.artifact.arguments;
  out->scalars.assign(args.size(), BoundParameters::Scalar{});
  std::size_t map_count = 0;
  for (const auto& a : args) map_count += a.source.kind == KernelArgumentSourceKind::kTensorMap ? 1 : 0;
  out->maps.assign(map_count, CUtensorMap{});
  out->pointers.assign(args.size(), nullptr);
  const Node& node = *context->node;
  std::size_t next_map = 0;
  int reserved_seen = 0;
  for (std::size_t i = 0; i < args.size(); ++i) {
    const KernelArgumentSource& s = args[i].source;
    BoundParameters::Scalar& slot = out->scalars[i];
    out->pointers[i] = &slot;
    const Tensor* tensor = nullptr;
    switch (s.kind) {
      case KernelArgumentSourceKind::kInput:
        CUTRITON_RETURN_IF_ERROR(TensorAt(inv.inputs, s.index, s.prepack, context, &tensor));
        slot.pointer = DeviceAddress(*tensor);
        break;
      case KernelArgumentSourceKind::kOutput:
        CUTRITON_RETURN_IF_ERROR(TensorAt(inv.outputs, s.index, "", context, &tensor));
        slot.pointer = DeviceAddress(*tensor);
        break;
      case KernelArgumentSourceKind::kInputDim:
      case KernelArgumentSourceKind::kOutputDim: {
        const bool in = s.kind == KernelArgumentSourceKind::kInputDim;
        CUTRITON_RETURN_IF_ERROR(TensorAt(in ? inv.inputs : inv.outputs, s.index, "", context, &tensor));
        const auto& shape = tensor->desc().shape;
        if (s.axis < 0 || static_cast<std::size_t>(s.axis) >= shape.size()) {
          return Status::ShapeError("kernel dimension axis is invalid");
        }
        CUTRITON_RETURN_IF_ERROR(Int32From(shape[static_cast<std::size_t>(s.axis)], "dimension", &slot.i32));
        break;
      }
      case KernelArgumentSourceKind::kInputDimProduct: {
        CUTRITON_RETURN_IF_ERROR(TensorAt(inv.inputs, s.index, "", context, &tensor));
        const auto& shape = tensor->desc().shape;
        if (s.begin_axis < 0 || static_cast<std::size_t>(s.begin_axis) > shape.size()) {
          return Status::ShapeError("kernel dimension product axis is invalid");
        }
        int64_t product = 1;
        for (std::size_t a = static_cast<std::size_t>(s.begin_axis); a < shape.size(); ++a) product *= shape[a];
        CUTRITON_RETURN_IF_ERROR(Int32From(product, "dimension product", &slot.i32));
        break;
      }
      case KernelArgumentSourceKind::kOutputNumElements:
      case KernelArgumentSourceKind::kInputNumElements: {
        const bool in = s.kind == KernelArgumentSourceKind::kInputNumElements;
        CUTRITON_RETURN_IF_ERROR(TensorAt(in ? inv.inputs : inv.outputs, s.index, "", context, &tensor));
        CUTRITON_RETURN_IF_ERROR(Int32From(tensor->desc().NumElements(), "element count", &slot.i32));
        break;
      }
      case KernelArgumentSourceKind::kAttributeInt64:
        slot.i32 = static_cast<int32_t>(AttributeInt(node, s));
        break;
      case KernelArgumentSourceKind::kAttributeFloat64:
        slot.f32 = static_cast<float>(AttributeFloat(node, s));
        break;
      case KernelArgumentSourceKind::kLiteralInt32:
        slot.i32 = static_cast<int32_t>(s.default_int);
        break;
      case KernelArgumentSourceKind::kRuntimeReserved:
        slot.pointer = reserved_seen++ == 0
                           ? static_cast<CUdeviceptr>(reinterpret_cast<std::uintptr_t>(context->runtime_scratch))
                           : 0;
        break;
      case KernelArgumentSourceKind::kTensorMap: {
        CUTRITON_RETURN_IF_ERROR(TensorAt(s.map_output ? inv.outputs : inv.inputs, s.index,
                                          s.map_output ? "" : s.prepack, context, &tensor));
        CUtensorMap* map = &out->maps[next_map++];
        CUTRITON_RETURN_IF_ERROR(EncodeTensorMap(*tensor, s, map));
        out->pointers[i] = map;
        break;
      }
    }
  }
  return Status::OK();
}

Status EvaluateGrid(const GridExpression& e, const KernelInvocation& inv, KernelContext* context, int sm_count,
                    int64_t* value) {
  auto tensor_of = [&](bool output, int index, const Tensor** t) -> Status {
    const auto& names = output ? inv.outputs : inv.inputs;
    if (index < 0 || static_cast<std::size_t>(index) >= names.size()) {
      return Status::InvalidArgument("launch-grid tensor index is invalid");
    }
    *t = FindTensor(context, names[static_cast<std::size_t>(index)]);
    return *t == nullptr ? Status::NotFound("launch-grid tensor is not bound") : Status::OK();
  };
  const Tensor* t = nullptr;
  switch (e.kind) {
    case GridExpressionKind::kLiteral:
      *value = e.literal;
      break;
    case GridExpressionKind::kVariantMeta: {
      const auto it = inv.artifact.launch_meta.find(e.meta_name);
      if (it == inv.artifact.launch_meta.end()) {
        return Status::InvalidArgument("launch grid references missing variant meta: " + e.meta_name);
      }
      *value = it->second;
      break;
    }
    case GridExpressionKind::kInputDim:
    case GridExpressionKind::kOutputDim: {
      CUTRITON_RETURN_IF_ERROR(tensor_of(e.kind == GridExpressionKind::kOutputDim, e.tensor_index, &t));
      const auto& shape = t->desc().shape;
      if (e.axis < 0 || static_cast<std::size_t>(e.axis) >= shape.size()) {
        return Status::ShapeError("launch-grid tensor axis is invalid");
      }
      *value = shape[static_cast<std::size_t>(e.axis)];
      break;
    }
    case GridExpressionKind::kInputNumElements:
    case GridExpressionKind::kOutputNumElements:
      CUTRITON_RETURN_IF_ERROR(tensor_of(e.kind == GridExpressionKind::kOutputNumElements, e.tensor_index, &t));
      *value = t->desc().NumElements();
      break;
    case GridExpressionKind::kDeviceSmCount:
      *value = sm_count;
      break;
    case GridExpressionKind::kCeilDiv:
    case GridExpressionKind::kMultiply:
    case GridExpressionKind::kMinimum: {
      if (e.operands.size() != 2) return Status::InvalidArgument("launch-grid binary expression is malformed");
      int64_t lhs = 0, rhs = 0;
      CUTRITON_RETURN_IF_ERROR(EvaluateGrid(e.operands[0], inv, context, sm_count, &lhs));
      CUTRITON_RETURN_IF_ERROR(EvaluateGrid(e.operands[1], inv, context, sm_count, &rhs));
      if (lhs <= 0 || rhs <= 0) return Status::ShapeError("launch-grid operands must be positive");
      if (e.kind == GridExpressionKind::kCeilDiv) {
        *value = (lhs + rhs - 1) / rhs;
      } else if (e.kind == GridExpressionKind::kMinimum) {
        *value = lhs < rhs ? lhs : rhs;
      } else {
        if (lhs > std::numeric_limits<int64_t>::max() / rhs) {
          return Status::ShapeError("launch-grid multiplication overflows");
        }
        *value = lhs * rhs;
      }
      break;
    }
  }
  return *value > 0 ? Status::OK() : Status::ShapeError("launch-grid dimension is not positive");
}

class InvocationKernel final : public OpKernel {
 public:
  InvocationKernel(KernelInvocation invocation, std::shared_ptr<CudaModuleCache> cache, CUfunction fn,
                   int sm_count)
      : invocation_(std::move(invocation)), cache_(std::move(cache)), function_(fn), sm_count_(sm_count) {}

  const char* backend_name() const override { return "cuda_sm100"; }
  const char* op_type() const override { return invocation_.artifact.op_type.c_str(); }

  Status Compute(KernelContext* context) override {
    if (context == nullptr || context->node == nullptr || context->tensors == nullptr) {
      return Status::InvalidArgument("invalid artifact kernel context");
    }
    CUTRITON_RETURN_IF_ERROR(BindArguments(invocation_, context, &params_));
    unsigned int grid[3] = {1, 1, 1};
    for (int axis = 0; axis < 3; ++axis) {
      int64_t extent = 0;
      CUTRITON_RETURN_IF_ERROR(
          EvaluateGrid(invocation_.artifact.launch_grid[axis], invocation_, context, sm_count_, &extent));
      const int64_t limit = axis == 0 ? 2147483647LL : 65535LL;
      if (extent > limit) return Status::ShapeError("launch-grid dimension exceeds CUDA limits");
      grid[axis] = static_cast<unsigned int>(extent);
    }
    const auto& a = invocation_.artifact;
    if (a.programmatic_launch) {
      // The kernel waits for its predecessor itself (griddepcontrol.wait), so
      // its CTAs may start on SMs the previous kernel has already left.
      CUlaunchAttribute attribute{};
      attribute.id = CU_LAUNCH_ATTRIBUTE_PROGRAMMATIC_STREAM_SERIALIZATION;
      attribute.value.programmaticStreamSerializationAllowed = 1;
      CUlaunchConfig config{};
      config.gridDimX = grid[0];
      config.gridDimY = grid[1];
      config.gridDimZ = grid[2];
      config.blockDimX = static_cast<unsigned int>(a.num_warps * 32);
      config.blockDimY = 1;
      config.blockDimZ = 1;
      config.sharedMemBytes = static_cast<unsigned int>(a.shared_memory_bytes);
      config.hStream = reinterpret_cast<CUstream>(context->stream);
      config.attrs = &attribute;
      config.numAttrs = 1;
      return drv::Check(drv::Get().cuLaunchKernelEx(&config, function_, params_.pointers.data(), nullptr),
                        "cuLaunchKernelEx");
    }
    return drv::Check(drv::Get().cuLaunchKernel(function_, grid[0], grid[1], grid[2],
                                                static_cast<unsigned int>(a.num_warps * 32), 1, 1,
                                                static_cast<unsigned int>(a.shared_memory_bytes),
                                                reinterpret_cast<CUstream>(context->stream),
                                                params_.pointers.data(), nullptr),
                      "cuLaunchKernel");
  }

 private:
  KernelInvocation invocation_;
  std::shared_ptr<CudaModuleCache> cache_;
  CUfunction function_{};
  int sm_count_{1};
  BoundParameters params_;
};

}  // namespace

Status CreateCudaModuleCache(int device_id, std::shared_ptr<CudaModuleCache>* cache) {
  if (cache == nullptr) return Status::InvalidArgument("module cache output is null");
  auto created = std::make_shared<CudaModuleCache>(device_id);
  CUTRITON_RETURN_IF_ERROR(created->Initialize());
  *cache = std::move(created);
  return Status::OK();
}

Status CreateInvocationKernel(const KernelInvocation& invocation, int device_id,
                              std::shared_ptr<CudaModuleCache> cache,
                              std::unique_ptr<OpKernel>* kernel) {
  if (kernel == nullptr || cache == nullptr) return Status::InvalidArgument("invocation kernel arguments are invalid");
  CUfunction function{};
  CUTRITON_RETURN_IF_ERROR(cache->GetFunction(invocation.artifact, &function));
  CUdevice device{};
  int sm_count = 0;
  const auto& api = drv::Get();
  CUTRITON_RETURN_IF_ERROR(drv::Check(api.cuDeviceGet(&device, device_id), "cuDeviceGet"));
  CUTRITON_RETURN_IF_ERROR(drv::Check(
      api.cuDeviceGetAttribute(&sm_count, CU_DEVICE_ATTRIBUTE_MULTIPROCESSOR_COUNT, device), "cuDeviceGetAttribute"));
  *kernel = std::make_unique<InvocationKernel>(invocation, std::move(cache), function, sm_count);
  return Status::OK();
}

std::size_t LoadedModuleCount(const std::shared_ptr<CudaModuleCache>& cache) {
  return cache == nullptr ? 0 : cache->size();
}

}  // namespace cutriton
