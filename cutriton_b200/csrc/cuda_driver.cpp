#include "cuda_driver.h"

#include <dlfcn.h>

#include <mutex>

namespace cutriton {
namespace drv {
namespace {

using GetProcAddressFn = CUresult (*)(const char*, void**, int, cuuint64_t,
                                      CUdriverProcAddressQueryResult*);

Api LoadApi() {
  Api api;
  void* handle = dlopen("libcuda.so.1", RTLD_NOW | RTLD_LOCAL);
  if (handle == nullptr) {
    api.load_error = std::string("libcuda.so.1 is not loadable: ") + dlerror();
    return api;
  }
  auto get_proc = reinterpret_cast<GetProcAddressFn>(dlsym(handle, "cuGetProcAddress_v2"));
  bool complete = true;
  auto resolve = [&](const char* name, const char* versioned, void** slot) {
    void* fn = nullptr;
    if (get_proc != nullptr) {
      CUdriverProcAddressQueryResult query{};
      if (get_proc(name, &fn, CUDA_VERSION, CU_GET_PROC_ADDRESS_DEFAULT, &query) != CUDA_SUCCESS ||
          query != CU_GET_PROC_ADDRESS_SUCCESS) {
        fn = nullptr;
      }
    }
    if (fn == nullptr) fn = dlsym(handle, versioned);
    if (fn == nullptr) {
      complete = false;
      api.load_error += std::string(" missing:") + name;
    }
    *slot = fn;
  };
#define CUTRITON_STRINGIFY2(x) #x
#define CUTRITON_STRINGIFY(x) CUTRITON_STRINGIFY2(x)
#define CUTRITON_RESOLVE_PFN(name) \
  resolve(#name, CUTRITON_STRINGIFY(name), reinterpret_cast<void**>(&api.name));
  CUTRITON_DRIVER_FUNCTIONS(CUTRITON_RESOLVE_PFN)
#undef CUTRITON_RESOLVE_PFN
  api.available = complete;
  return api;
}

}  // namespace

const Api& Get() {
  static const Api api = LoadApi();
  return api;
}

Status Ensure() {
  const Api& api = Get();
  if (!api.available) {
    return Status::RuntimeError("CUDA driver unavailable:" + api.load_error);
  }
  static std::once_flag once;
  static CUresult init_result = CUDA_SUCCESS;
  std::call_once(once, [&]() { init_result = api.cuInit(0); });
  return Check(init_result, "cuInit");
}

Status Check(CUresult result, const char* operation) {
  if (result == CUDA_SUCCESS) return Status::OK();
  const Api& api = Get();
  const char* name = nullptr;
  const char* text = nullptr;
  if (api.cuGetErrorName != nullptr) api.cuGetErrorName(result, &name);
  if (api.cuGetErrorString != nullptr) api.cuGetErrorString(result, &text);
  return Status::RuntimeError(std::string(operation) + " failed: " +
                              (name ? name : "CUDA_ERROR") + " (" +
                              (text ? text : "unknown") + ")");
}

Status RetainPrimaryContext(int device_id, CUdevice* device, CUcontext* context) {
  CUTRITON_RETURN_IF_ERROR(Ensure());
  const Api& api = Get();
  CUTRITON_RETURN_IF_ERROR(Check(api.cuDeviceGet(device, device_id), "cuDeviceGet"));
  CUTRITON_RETURN_IF_ERROR(
      Check(api.cuDevicePrimaryCtxRetain(context, *device), "cuDevicePrimaryCtxRetain"));
  Status status = Check(api.cuCtxSetCurrent(*context), "cuCtxSetCurrent");
  if (!status.ok()) api.cuDevicePrimaryCtxRelease(*device);
  return status;
}

Status ComputeCapability(int device_id, int* capability) {
  CUTRITON_RETURN_IF_ERROR(Ensure());
  const Api& api = Get();
  CUdevice device{};
  CUTRITON_RETURN_IF_ERROR(Check(api.cuDeviceGet(&device, device_id), "cuDeviceGet"));
  int major = 0, minor = 0;
  CUTRITON_RETURN_IF_ERROR(Check(api.cuDeviceGetAttribute(
      &major, CU_DEVICE_ATTRIBUTE_COMPUTE_CAPABILITY_MAJOR, device), "cuDeviceGetAttribute"));
  CUTRITON_RETURN_IF_ERROR(Check(api.cuDeviceGetAttribute(
      &minor, CU_DEVICE_ATTRIBUTE_COMPUTE_CAPABILITY_MINOR, device), "cuDeviceGetAttribute"));
  *capability = major * 10 + minor;
  return Status::OK();
}

}  // namespace drv
}  // namespace cutriton
