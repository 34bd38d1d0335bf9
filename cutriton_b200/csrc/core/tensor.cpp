#include "cutriton/core/tensor.h"

#include <limits>

namespace cutriton {

const char* DataTypeName(DataType dtype) {
  switch (dtype) {
    case DataType::kFloat32: return "float32";
    case DataType::kFloat16: return "float16";
    case DataType::kInt32: return "int32";
    case DataType::kInt64: return "int64";
    case DataType::kUnknown: break;
  }
  return "unknown";
}

const char* DeviceTypeName(DeviceType device_type) {
  return device_type == DeviceType::kCUDA ? "cuda" : "cpu";
}

std::size_t ElementSize(DataType dtype) {
  switch (dtype) {
    case DataType::kFloat32:
    case DataType::kInt32: return 4;
    case DataType::kFloat16: return 2;
    case DataType::kInt64: return 8;
    case DataType::kUnknown: break;
  }
  return 0;
}

bool TensorDesc::IsStatic() const {
  if (shape.empty() || dtype == DataType::kUnknown) return false;
  for (int64_t dim : shape) {
    if (dim <= 0) return false;
  }
  return true;
}

int64_t TensorDesc::NumElements() const {
  if (shape.empty()) return 0;
  int64_t count = 1;
  for (int64_t dim : shape) {
    if (dim <= 0 || count > std::numeric_limits<int64_t>::max() / dim) return 0;
    count *= dim;
  }
  return count;
}

std::size_t TensorDesc::ByteSize() const {
  const int64_t count = NumElements();
  const std::size_t element = ElementSize(dtype);
  return (count <= 0 || element == 0) ? 0 : static_cast<std::size_t>(count) * element;
}

Status TensorDesc::Validate() const {
  if (dtype == DataType::kUnknown) return Status::ShapeError("tensor dtype is unknown");
  if (shape.empty()) return Status::ShapeError("tensor shape is empty");
  for (int64_t dim : shape) {
    if (dim <= 0) return Status::ShapeError("static tensor shape has a non-positive dimension");
  }
  if (ByteSize() == 0) return Status::ShapeError("tensor byte size is zero");
  return Status::OK();
}

}  // namespace cutriton
