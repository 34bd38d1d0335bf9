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
// Programmatic dependent launch. Every pack kernel (launched with
// programmatic stream serialization, see cuda_launcher.cpp) first lets the
// next kernel start launching, then waits until the preceding kernel in the
// stream has completed and its writes are visible. Nothing before the wait
// may touch activation memory (reads or writes): only shared memory, TMEM and
// kernel parameters. Without the launch attribute both are no-ops.
#define CTB_GRID_DEPENDENCY_SYNC()                                      \
  do {                                                                  \
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");     \
    asm volatile("griddepcontrol.wait;" ::: "memory");                  \
  } while (0)

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

// erf(z) by Abramowitz & Stegun, Handbook of Mathematical Functions, formula
// 7.1.26: erf(z) = 1 - (a1 t + a2 t^2 + a3 t^3 + a4 t^4 + a5 t^5) exp(-z^2),
// t = 1 / (1 + p z) for z >= 0 (odd extension below), |error| <= 1.5e-7 —
// far below the FP16 rounding of the GEMM epilogue that uses it, at a third
// of the instructions of erff (one reciprocal, one exp, five FMAs).
__device__ __forceinline__ float erf_as7126(float z) {
  const float a = fabsf(z);
  const float t = __fdividef(1.0f, fmaf(0.3275911f, a, 1.0f));
  float poly = fmaf(1.061405429f, t, -1.453152027f);
  poly = fmaf(poly, t, 1.421413741f);
  poly = fmaf(poly, t, -0.284496736f);
  poly = fmaf(poly, t, 0.254829592f);
  poly *= t;
  const float r = fmaf(-poly, __expf(-a * a), 1.0f);
  return copysignf(r, z);
}

// GELU with erf_as7126 (max deviation from the exact-erf GELU 1.1e-7 |x|).
__device__ __forceinline__ float gelu_erf_fast(float x) {
  return 0.5f * x * (1.0f + erf_as7126(x * 0.7071067811865476f));
}

}  // namespace ctb
