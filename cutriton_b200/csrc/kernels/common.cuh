// Shared device helpers for the sm_100a Kernel Pack.
//
// Every pack kernel ends its parameter list with two runtime_reserved
// pointers (pack ABI). The engine binds the first to the context's error
// block; kernels with bounded spin-waits record an expired wait there and
// return instead of hanging. The second is reserved (always null).
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

#define CTB_RESERVED_PARAMS void* runtime_scratch, void* profile_scratch
#define CTB_UNUSED_RESERVED() \
  do {                        \
    (void)runtime_scratch;    \
    (void)profile_scratch;    \
  } while (0)

namespace ctb {

// Matches ErrorBlock in runtime/engine.cpp.
struct ErrorBlock {
  unsigned int code;
  unsigned int site;
  unsigned int block;
  unsigned int reserved[13];
};

// Error codes written by kernels.
enum : unsigned int {
  kErrorWaitTimeout = 1,  // a bounded mbarrier / flag wait expired
  kErrorBadShape = 2,     // the kernel met a shape outside its contract
};

__device__ __forceinline__ void report_error(void* scratch, unsigned int code, unsigned int site) {
  if (scratch == nullptr) return;
  ErrorBlock* e = static_cast<ErrorBlock*>(scratch);
  if (atomicCAS(&e->code, 0u, code) == 0u) {
    e->site = site;
    e->block = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z);
    __threadfence_system();
  }
}

__device__ __forceinline__ bool aligned16(const void* p) {
  return (reinterpret_cast<uintptr_t>(p) & 15u) == 0;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int offset = 16; offset > 0; offset >>= 1) v += __shfl_xor_sync(0xffffffffu, v, offset);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int offset = 16; offset > 0; offset >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, offset));
  return v;
}

// Exact GELU, 0.5 x (1 + erf(x / sqrt 2)), on an FP32 value (CUDA erff).
__device__ __forceinline__ float gelu_erf(float x) {
  return 0.5f * x * (1.0f + erff(x * 0.7071067811865476f));
}

}  // namespace ctb
