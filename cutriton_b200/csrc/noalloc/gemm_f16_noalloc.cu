// ctb_gemm_f16_noalloc: the persistent FP16 GEMM (kernels/gemm_f16_tp.cu) as
// a single C call that allocates no device or pinned memory.
//
// Who needs it: callers that must not allocate on the call path — a serving
// loop that has fixed its memory footprint up front, a host whose allocator is
// locked down, or code running while a device-wide allocation would
// serialise against other work. The engine path binds the kernel's scratch
// (its error block) to a context-owned buffer; here that scratch lives in
// this file's static __device__ array instead, so nothing is allocated per
// call or per device.
//
// Contract:
//   * scratch: g_noalloc_scratch, kNoAllocScratchBytes (256) per device; the
//     GEMM needs sizeof(ErrorBlock) = 64 of it. A kernel whose scratch need
//     exceeds the array is rejected with an error message, not launched.
//   * what must start at zero: the error block. Every call clears it
//     (cudaMemsetAsync on the caller's stream) before the launch.
//   * the first call on a device does the set-up (symbol address, SM count,
//     shared-memory opt-in, driver entry point) with that device current; make
//     that first call before any stream capture.
//   * calls that overlap in time on one device (different host threads or
//     streams) share the scratch array and race on it: serialise them.
//   * operands: A [m, k] and B^T [n, k] row-major FP16 (B already transposed:
//     the engine's "transpose_2d" prepack), C [m, n] FP16; k and n multiples
//     of 8; all three 16-byte aligned. The call is synchronous on `stream`
//     (it reads the error block back) and returns 0 on success.

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdio>
#include <cstring>
#include <mutex>

#include "../kernels/gemm_f16_tp.cu"
#include "cutriton_b200_noalloc.h"

namespace {

constexpr size_t kNoAllocScratchBytes = 256;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
constexpr int kSmemBytes = 196608 + 32768 + 256 + 1024;  // ring + staging + barriers + alignment

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

struct DeviceSetup {
  bool ready = false;
  void* scratch = nullptr;
  int sm_count = 0;
};

DeviceSetup g_devices[kMaxDevices];
EncodeTiledFn g_encode = nullptr;
std::mutex g_setup_mutex;

int Fail(char* error, size_t error_len, int code, const char* message) {
  if (error != nullptr && error_len > 0) std::snprintf(error, error_len, "%s", message);
  return code;
}

int FailCuda(char* error, size_t error_len, const char* what, cudaError_t status) {
  char message[256];
  std::snprintf(message, sizeof(message), "%s failed: %s", what, cudaGetErrorString(status));
  return Fail(error, error_len, CTB_NOALLOC_CUDA_ERROR, message);
}

// Row-major [rows, cols] FP16 matrix, box {box_cols columns, box_rows rows}:
// operands 64 x 128 with a 128-byte swizzle, the output store box 32 x 32
// with a 64-byte swizzle (the kernel's staging layout).
bool EncodeFp16(CUtensorMap* map, const void* base, int rows, int cols, int box_cols, int box_rows,
                CUtensorMapSwizzle swizzle) {
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(cols) * 2};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(box_cols), static_cast<cuuint32_t>(box_rows)};
  const cuuint32_t element_strides[2] = {1, 1};
  return g_encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box,
                  element_strides, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

extern "C" int ctb_gemm_f16_noalloc(const void* a, const void* b_t, void* c, int m, int n, int k, int apply_gelu,
                                    void* stream, char* error, size_t error_len) {
  if (a == nullptr || b_t == nullptr || c == nullptr) {
    return Fail(error, error_len, CTB_NOALLOC_INVALID_ARGUMENT, "A, B^T and C must be device pointers");
  }
  if (m <= 0 || n <= 0 || k <= 0 || k % 8 != 0 || n % 8 != 0) {
    return Fail(error, error_len, CTB_NOALLOC_INVALID_ARGUMENT, "need m, n, k > 0 with k and n multiples of 8");
  }
  if (((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b_t) | reinterpret_cast<uintptr_t>(c)) & 15) !=
      0) {
    return Fail(error, error_len, CTB_NOALLOC_INVALID_ARGUMENT, "A, B^T and C must be 16-byte aligned");
  }
  const size_t scratch_needed = sizeof(ctb::ErrorBlock);
  if (scratch_needed > kNoAllocScratchBytes) {
    return Fail(error, error_len, CTB_NOALLOC_SCRATCH_TOO_SMALL,
                "the kernel needs more scratch than the 256-byte static array holds");
  }

  int device = 0;
  cudaError_t status = cudaGetDevice(&device);
  if (status != cudaSuccess) return FailCuda(error, error_len, "cudaGetDevice", status);
  if (device < 0 || device >= kMaxDevices) {
    return Fail(error, error_len, CTB_NOALLOC_INVALID_ARGUMENT, "device ordinal out of range");
  }
  if (stream != nullptr) {
    // The scratch address, SM count and shared-memory opt-in below belong to
    // the current device; a stream of another device would get the wrong ones.
    int stream_device = -1;
    status = cudaStreamGetDevice(static_cast<cudaStream_t>(stream), &stream_device);
    if (status != cudaSuccess) return FailCuda(error, error_len, "cudaStreamGetDevice", status);
    if (stream_device != device) {
      char message[160];
      std::snprintf(message, sizeof(message), "stream belongs to device %d but device %d is current",
                    stream_device, device);
      return Fail(error, error_len, CTB_NOALLOC_INVALID_ARGUMENT, message);
    }
  }
  DeviceSetup& setup = g_devices[device];
  {
    // Once per device, with that device current (it is: cudaGetDevice above).
    std::lock_guard<std::mutex> lock(g_setup_mutex);
    if (!setup.ready) {
      status = cudaGetSymbolAddress(&setup.scratch, g_noalloc_scratch);
      if (status != cudaSuccess) return FailCuda(error, error_len, "cudaGetSymbolAddress", status);
      status = cudaDeviceGetAttribute(&setup.sm_count, cudaDevAttrMultiProcessorCount, device);
      if (status != cudaSuccess) return FailCuda(error, error_len, "cudaDeviceGetAttribute", status);
      for (const void* fn : {reinterpret_cast<const void*>(ctb_gemm_f16_tp),
                             reinterpret_cast<const void*>(ctb_gemm_gelu_f16_tp)}) {
        status = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
        if (status != cudaSuccess) return FailCuda(error, error_len, "cudaFuncSetAttribute", status);
      }
      if (g_encode == nullptr) {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult found{};
        status = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &found);
        if (status != cudaSuccess || found != cudaDriverEntryPointSuccess || fn == nullptr) {
          return Fail(error, error_len, CTB_NOALLOC_CUDA_ERROR, "cuTensorMapEncodeTiled is not available");
        }
        g_encode = reinterpret_cast<EncodeTiledFn>(fn);
      }
      setup.ready = true;
    }
  }

  // Host-side descriptors (passed by value as __grid_constant__ parameters).
  ctb::tc::TmaDescriptor tma_a, tma_b, tma_out;
  if (!EncodeFp16(reinterpret_cast<CUtensorMap*>(&tma_a), a, m, k, 64, 128, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !EncodeFp16(reinterpret_cast<CUtensorMap*>(&tma_b), b_t, n, k, 64, 128, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !EncodeFp16(reinterpret_cast<CUtensorMap*>(&tma_out), c, m, n, kChunk, 32, CU_TENSOR_MAP_SWIZZLE_64B)) {
    return Fail(error, error_len, CTB_NOALLOC_CUDA_ERROR, "cuTensorMapEncodeTiled rejected an operand");
  }
  const auto s = static_cast<cudaStream_t>(stream);
  // The error block must start at zero.
  status = cudaMemsetAsync(setup.scratch, 0, scratch_needed, s);
  if (status != cudaSuccess) return FailCuda(error, error_len, "cudaMemsetAsync", status);
  const long long tiles = static_cast<long long>((m + 127) / 128) * ((n + 127) / 128);
  const unsigned grid = static_cast<unsigned>(tiles < setup.sm_count ? tiles : setup.sm_count);
  __half* out = static_cast<__half*>(c);
  if (apply_gelu) {
    ctb_gemm_gelu_f16_tp<<<grid, kThreads, kSmemBytes, s>>>(tma_a, tma_b, tma_out, out, m, n, k, setup.scratch, nullptr);
  } else {
    ctb_gemm_f16_tp<<<grid, kThreads, kSmemBytes, s>>>(tma_a, tma_b, tma_out, out, m, n, k, setup.scratch, nullptr);
  }
  status = cudaGetLastError();
  if (status != cudaSuccess) return FailCuda(error, error_len, "kernel launch", status);
  ctb::ErrorBlock reported{};
  status = cudaMemcpyAsync(&reported, setup.scratch, sizeof(reported), cudaMemcpyDeviceToHost, s);
  if (status != cudaSuccess) return FailCuda(error, error_len, "cudaMemcpyAsync", status);
  status = cudaStreamSynchronize(s);
  if (status != cudaSuccess) return FailCuda(error, error_len, "cudaStreamSynchronize", status);
  if (reported.code != 0) {
    char message[160];
    std::snprintf(message, sizeof(message), "the kernel abandoned a bounded wait (code %u, site %u, block %u)",
                  reported.code, reported.site, reported.block);
    return Fail(error, error_len, CTB_NOALLOC_KERNEL_ERROR, message);
  }
  return CTB_NOALLOC_OK;
}
