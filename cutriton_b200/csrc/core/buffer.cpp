#include "cutriton/core/buffer.h"

#include <cstring>

#include "../cuda_driver.h"

namespace cutriton {
namespace {

// Keeps the primary context retained for the lifetime of a scope.
class ScopedPrimaryContext {
 public:
  Status Enter(int device_id) {
    status_ = drv::RetainPrimaryContext(device_id, &device_, &context_);
    return status_;
  }
  ~ScopedPrimaryContext() {
    if (status_.ok() && context_ != nullptr) drv::Get().cuDevicePrimaryCtxRelease(device_);
  }

 private:
  Status status_{ErrorCode::kInternal, "not entered"};
  CUdevice device_{};
  CUcontext context_{};
};

Status CheckRange(std::size_t capacity, std::size_t offset, std::size_t size,
                  const char* what) {
  if (offset > capacity || size > capacity - offset) {
    return Status::InvalidArgument(std::string("buffer copy exceeds ") + what + " capacity");
  }
  return Status::OK();
}

}  // namespace

std::shared_ptr<Buffer> Buffer::AllocateHost(std::size_t size_bytes) {
  if (size_bytes == 0) return std::make_shared<Buffer>();
  auto* raw = new std::uint8_t[size_bytes]();
  std::shared_ptr<void> owner(raw, [](void* p) { delete[] static_cast<std::uint8_t*>(p); });
  return std::shared_ptr<Buffer>(new Buffer(raw, size_bytes, DeviceType::kCPU, 0, owner));
}

Status Buffer::AllocateCuda(std::size_t size_bytes, int device_id,
                            std::shared_ptr<Buffer>* buffer) {
  if (buffer == nullptr) return Status::InvalidArgument("CUDA buffer output pointer is null");
  if (size_bytes == 0) {
    *buffer = std::make_shared<Buffer>();
    return Status::OK();
  }
  CUdevice device{};
  CUcontext context{};
  CUTRITON_RETURN_IF_ERROR(drv::RetainPrimaryContext(device_id, &device, &context));
  const auto& api = drv::Get();
  CUdeviceptr pointer{};
  Status status = drv::Check(api.cuMemAlloc(&pointer, size_bytes), "cuMemAlloc");
  if (!status.ok()) {
    api.cuDevicePrimaryCtxRelease(device);
    return status;
  }
  void* raw = reinterpret_cast<void*>(static_cast<std::uintptr_t>(pointer));
  // The retained primary context is held by the allocation and released with it.
  std::shared_ptr<void> owner(raw, [device, context](void* p) {
    const auto& d = drv::Get();
    if (d.cuCtxSetCurrent(context) == CUDA_SUCCESS) {
      d.cuMemFree(static_cast<CUdeviceptr>(reinterpret_cast<std::uintptr_t>(p)));
    }
    d.cuDevicePrimaryCtxRelease(device);
  });
  *buffer = std::shared_ptr<Buffer>(
      new Buffer(raw, size_bytes, DeviceType::kCUDA, device_id, std::move(owner)));
  return Status::OK();
}

std::shared_ptr<Buffer> Buffer::WrapExternal(void* data, std::size_t size_bytes,
                                             DeviceType device_type, int device_id) {
  return std::shared_ptr<Buffer>(new Buffer(data, size_bytes, device_type, device_id, nullptr));
}

Status Buffer::CopyFromHost(const void* source, std::size_t size_bytes,
                            std::size_t destination_offset) {
  if (source == nullptr && size_bytes != 0) return Status::InvalidArgument("host source pointer is null");
  CUTRITON_RETURN_IF_ERROR(CheckRange(size_bytes_, destination_offset, size_bytes, "destination"));
  if (size_bytes == 0) return Status::OK();
  if (device_type_ == DeviceType::kCPU) {
    std::memcpy(static_cast<std::uint8_t*>(data_) + destination_offset, source, size_bytes);
    return Status::OK();
  }
  ScopedPrimaryContext scope;
  CUTRITON_RETURN_IF_ERROR(scope.Enter(device_id_));
  const CUdeviceptr destination =
      static_cast<CUdeviceptr>(reinterpret_cast<std::uintptr_t>(data_)) + destination_offset;
  return drv::Check(drv::Get().cuMemcpyHtoD(destination, source, size_bytes), "cuMemcpyHtoD");
}

Status Buffer::CopyToHost(void* destination, std::size_t size_bytes,
                          std::size_t source_offset) const {
  if (destination == nullptr && size_bytes != 0) return Status::InvalidArgument("host destination pointer is null");
  CUTRITON_RETURN_IF_ERROR(CheckRange(size_bytes_, source_offset, size_bytes, "source"));
  if (size_bytes == 0) return Status::OK();
  if (device_type_ == DeviceType::kCPU) {
    std::memcpy(destination, static_cast<const std::uint8_t*>(data_) + source_offset, size_bytes);
    return Status::OK();
  }
  ScopedPrimaryContext scope;
  CUTRITON_RETURN_IF_ERROR(scope.Enter(device_id_));
  const CUdeviceptr source =
      static_cast<CUdeviceptr>(reinterpret_cast<std::uintptr_t>(data_)) + source_offset;
  return drv::Check(drv::Get().cuMemcpyDtoH(destination, source, size_bytes), "cuMemcpyDtoH");
}

}  // namespace cutriton
