#pragma once

// Host or device byte range, owned (with a deleter) or wrapped (API of the
// reference's include/cutriton/core/buffer.h:13-53). CUDA allocations go
// through the driver API on the device's primary context.

#include <cstddef>
#include <cstdint>
#include <memory>
#include <utility>

#include "cutriton/core/status.h"
#include "cutriton/core/tensor.h"

namespace cutriton {

class Buffer {
 public:
  Buffer() = default;
  // Zero-initialised host bytes.
  static std::shared_ptr<Buffer> AllocateHost(std::size_t size_bytes);
  // Device bytes on `device_id` (cuMemAlloc in the primary context).
  static Status AllocateCuda(std::size_t size_bytes, int device_id,
                             std::shared_ptr<Buffer>* buffer);
  // Non-owning view of memory that outlives the Buffer.
  static std::shared_ptr<Buffer> WrapExternal(void* data, std::size_t size_bytes,
                                              DeviceType device_type,
                                              int device_id = 0);
  Status CopyFromHost(const void* source, std::size_t size_bytes,
                      std::size_t destination_offset = 0);
  Status CopyToHost(void* destination, std::size_t size_bytes,
                    std::size_t source_offset = 0) const;

  void* data() const { return data_; }
  std::size_t size_bytes() const { return size_bytes_; }
  DeviceType device_type() const { return device_type_; }
  int device_id() const { return device_id_; }
  bool owns_memory() const { return owner_ != nullptr; }
  bool empty() const { return data_ == nullptr || size_bytes_ == 0; }

 private:
  Buffer(void* data, std::size_t size_bytes, DeviceType device_type,
         int device_id, std::shared_ptr<void> owner)
      : data_(data), size_bytes_(size_bytes), device_type_(device_type),
        device_id_(device_id), owner_(std::move(owner)) {}

  void* data_{nullptr};
  std::size_t size_bytes_{0};
  DeviceType device_type_{DeviceType::kCPU};
  int device_id_{0};
  std::shared_ptr<void> owner_;
};

}  // namespace cutriton
