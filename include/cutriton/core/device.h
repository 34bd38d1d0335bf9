#pragma once

// Device identity (API of the reference's include/cutriton/core/device.h:9-25).

#include <cstddef>
#include <string>

#include "cutriton/core/tensor.h"

namespace cutriton {

struct Device {
  DeviceType type{DeviceType::kCPU};
  int id{0};
  std::string name{"cpu"};

  static Device CPU() { return Device{}; }
  static Device CUDA(int device_id = 0) {
    return Device{DeviceType::kCUDA, device_id, "cuda:" + std::to_string(device_id)};
  }
};

struct DeviceProperties {
  Device device;
  int sm_count{0};
  std::size_t l2_cache_bytes{0};
  std::size_t global_memory_bytes{0};
};

}  // namespace cutriton
