#pragma once

// Tensor descriptions and views (API of the reference's
// include/cutriton/core/tensor.h:14-81). A Tensor is a description plus a
// shared Buffer and a byte offset into it; several Tensors may view one Buffer.

#include <cstddef>
#include <cstdint>
#include <memory>
#include <string>
#include <utility>
#include <vector>

#include "cutriton/core/status.h"

namespace cutriton {

enum class DataType {
  kUnknown = 0,
  kFloat32,
  kFloat16,
  kInt32,
  kInt64,
};

enum class DeviceType {
  kCPU = 0,
  kCUDA,
};

const char* DataTypeName(DataType dtype);
const char* DeviceTypeName(DeviceType device_type);
std::size_t ElementSize(DataType dtype);

struct TensorDesc {
  std::vector<int64_t> shape;
  DataType dtype{DataType::kUnknown};
  DeviceType device_type{DeviceType::kCPU};
  int device_id{0};
  std::string layout{"NCHW"};

  TensorDesc() = default;
  TensorDesc(std::vector<int64_t> dims, DataType type,
             DeviceType device = DeviceType::kCPU, int id = 0,
             std::string tensor_layout = "NCHW")
      : shape(std::move(dims)), dtype(type), device_type(device),
        device_id(id), layout(std::move(tensor_layout)) {}

  // True when every dimension is known (>0) and the dtype is known.
  bool IsStatic() const;
  // Product of the dimensions; 0 for empty, dynamic or overflowing shapes.
  int64_t NumElements() const;
  std::size_t ByteSize() const;
  Status Validate() const;
};

class Buffer;

class Tensor {
 public:
  Tensor() = default;
  Tensor(TensorDesc desc, std::shared_ptr<Buffer> buffer,
         std::size_t byte_offset = 0)
      : desc_(std::move(desc)), buffer_(std::move(buffer)),
        byte_offset_(byte_offset) {}

  const TensorDesc& desc() const { return desc_; }
  TensorDesc& mutable_desc() { return desc_; }
  const std::shared_ptr<Buffer>& buffer() const { return buffer_; }
  std::size_t byte_offset() const { return byte_offset_; }
  bool defined() const { return buffer_ != nullptr; }

 private:
  TensorDesc desc_;
  std::shared_ptr<Buffer> buffer_;
  std::size_t byte_offset_{0};
};

}  // namespace cutriton
