#pragma once

// Lazily loaded CUDA driver API table.
//
// The library resolves libcuda.so.1 at first use (dlopen + cuGetProcAddress at
// the CUDA_VERSION the headers describe) instead of linking it, so the shared
// library loads on hosts without an NVIDIA driver: every graph/IR/planning
// call works there, and device calls return kRuntimeError naming the missing
// driver. Only the types and prototypes of <cuda.h> are used.

#include <cuda.h>

#include <string>

#include "cutriton/core/status.h"

namespace cutriton {
namespace drv {

#define CUTRITON_DRIVER_FUNCTIONS(X) \
  X(cuInit)                          \
  X(cuDriverGetVersion)              \
  X(cuDeviceGet)                     \
  X(cuDeviceGetCount)                \
  X(cuDeviceGetAttribute)            \
  X(cuDeviceGetUuid)                 \
  X(cuDevicePrimaryCtxRetain)        \
  X(cuDevicePrimaryCtxRelease)       \
  X(cuCtxSetCurrent)                 \
  X(cuCtxGetCurrent)                 \
  X(cuMemAlloc)                      \
  X(cuMemFree)                       \
  X(cuMemcpyHtoD)                    \
  X(cuMemcpyDtoH)                    \
  X(cuMemsetD32Async)                \
  X(cuModuleLoadData)                \
  X(cuModuleUnload)                  \
  X(cuModuleGetFunction)             \
  X(cuFuncSetAttribute)              \
  X(cuLaunchKernel)                  \
  X(cuLaunchKernelEx)                \
  X(cuStreamCreate)                  \
  X(cuStreamDestroy)                 \
  X(cuStreamSynchronize)             \
  X(cuStreamBeginCapture)            \
  X(cuStreamEndCapture)              \
  X(cuGraphInstantiateWithFlags)     \
  X(cuGraphLaunch)                   \
  X(cuGraphExecDestroy)              \
  X(cuGraphDestroy)                  \
  X(cuEventCreate)                   \
  X(cuEventDestroy)                  \
  X(cuEventRecord)                   \
  X(cuEventRecordWithFlags)          \
  X(cuEventSynchronize)              \
  X(cuEventElapsedTime)              \
  X(cuGetErrorName)                  \
  X(cuGetErrorString)                \
  X(cuTensorMapEncodeTiled)          \
  X(cuMemHostAlloc)                  \
  X(cuMemHostGetDevicePointer)       \
  X(cuMemFreeHost)                   \
  X(cuMemcpyHtoDAsync)               \
  X(cuMemcpyDtoHAsync)

struct Api {
#define CUTRITON_DECLARE_PFN(name) decltype(&::name) name = nullptr;
  CUTRITON_DRIVER_FUNCTIONS(CUTRITON_DECLARE_PFN)
#undef CUTRITON_DECLARE_PFN
  bool available = false;
  std::string load_error;
};

// Loads the table once (thread-safe). `available` is false when the driver
// library or any entry point is missing.
const Api& Get();

// Ok() when the driver is loaded and cuInit succeeded.
Status Ensure();

// Maps a CUresult to Status::RuntimeError("<op> failed: NAME (string)").
Status Check(CUresult result, const char* operation);

// Retains the primary context of `device_id` and makes it current.
Status RetainPrimaryContext(int device_id, CUdevice* device, CUcontext* context);

// Compute capability as major*10+minor.
Status ComputeCapability(int device_id, int* capability);

}  // namespace drv
}  // namespace cutriton
