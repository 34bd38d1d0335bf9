// Row kernels over [rows, columns] FP16 (columns <= 1024): LayerNormalization,
// SkipLayerNormalization and Softmax along the last axis.
//
// One warp per row with the whole row held in registers (<= 32 values per
// lane), so each element is read once and written once. When the row length
// is a multiple of 8 (and rows are 16-byte aligned) every access is a 16-byte
// vector: lane owns columns 256 j + 8 lane .. + 7, so one warp instruction
// moves 512 contiguous bytes; otherwise lane owns columns lane + 32 j. Numerics follow
// python/cutriton/triton_kernels/transformer.py:128-190: FP32 math, mean
// first, then the variance of the centred values (two passes over registers),
// rsqrt(var + eps), gamma/beta widened from FP16; SkipLayerNormalization adds
// input and residual in FP32 before normalising.

#include "common.cuh"

namespace {

constexpr int kMaxPerLane = 32;  // 32 lanes x 32 = 1024 columns

// Loads row `row` of `src` widened to FP32: lane owns columns lane + 32*j.
__device__ __forceinline__ void load_row(const __half* __restrict__ src, int columns, float (&v)[kMaxPerLane]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int j = 0; j < kMaxPerLane; ++j) {
    const int col = lane + 32 * j;
    v[j] = col < columns ? __half2float(src[col]) : 0.0f;
  }
}

// Vector layout: v[8 j + e] = column 256 j + 8 lane + e.
__device__ __forceinline__ void load_row_vec(const __half* __restrict__ src, int columns, float (&v)[kMaxPerLane]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int j = 0; j < kMaxPerLane / 8; ++j) {
    const int col = 256 * j + 8 * lane;
    uint4 raw = make_uint4(0, 0, 0, 0);
    if (col < columns) raw = __ldg(reinterpret_cast<const uint4*>(src + col));
    const __half2* h = reinterpret_cast<const __half2*>(&raw);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = __half22float2(h[e]);
      v[8 * j + 2 * e] = f.x;
      v[8 * j + 2 * e + 1] = f.y;
    }
  }
}

__device__ __forceinline__ void normalize_row_vec(float (&v)[kMaxPerLane], int columns, float epsilon,
                                                  const __half* __restrict__ scale,
                                                  const __half* __restrict__ bias, __half* __restrict__ dst) {
  const int lane = threadIdx.x & 31;
  float sum = 0.0f;
#pragma unroll
  for (int j = 0; j < kMaxPerLane; ++j) sum += v[j];
  const float mean = ctb::warp_sum(sum) / static_cast<float>(columns);
  float squares = 0.0f;
#pragma unroll
  for (int j = 0; j < kMaxPerLane; ++j) {
    const int col = 256 * (j / 8) + 8 * lane;
    v[j] = col < columns ? v[j] - mean : 0.0f;
    squares += v[j] * v[j];
  }
  const float variance = ctb::warp_sum(squares) / static_cast<float>(columns);
  const float inv_std = rsqrtf(variance + epsilon);
#pragma unroll
  for (int j = 0; j < kMaxPerLane / 8; ++j) {
    const int col = 256 * j + 8 * lane;
    if (col < columns) {
      const uint4 g = __ldg(reinterpret_cast<const uint4*>(scale + col));
      const uint4 b = __ldg(reinterpret_cast<const uint4*>(bias + col));
      const __half2* gh = reinterpret_cast<const __half2*>(&g);
      const __half2* bh = reinterpret_cast<const __half2*>(&b);
      uint4 packed;
      __half2* o = reinterpret_cast<__half2*>(&packed);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 gf = __half22float2(gh[e]);
        const float2 bf = __half22float2(bh[e]);
        o[e] = __floats2half2_rn(v[8 * j + 2 * e] * inv_std * gf.x + bf.x,
                                 v[8 * j + 2 * e + 1] * inv_std * gf.y + bf.y);
      }
      *reinterpret_cast<uint4*>(dst + col) = packed;
    }
  }
}

__device__ __forceinline__ bool vector_rows(const void* a, const void* b, int columns) {
  return columns % 8 == 0 && ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b)) & 15) == 0;
}

__device__ __forceinline__ void normalize_row(float (&v)[kMaxPerLane], int columns, float epsilon,
                                              const __half* __restrict__ scale,
                                              const __half* __restrict__ bias, __half* __restrict__ dst) {
  const int lane = threadIdx.x & 31;
  float sum = 0.0f;
#pragma unroll
  for (int j = 0; j < kMaxPerLane; ++j) sum += v[j];
  const float mean = ctb::warp_sum(sum) / static_cast<float>(columns);
  float squares = 0.0f;
#pragma unroll
  for (int j = 0; j < kMaxPerLane; ++j) {
    const int col = lane + 32 * j;
    v[j] = col < columns ? v[j] - mean : 0.0f;
    squares += v[j] * v[j];
  }
  const float variance = ctb::warp_sum(squares) / static_cast<float>(columns);
  const float inv_std = rsqrtf(variance + epsilon);
#pragma unroll
  for (int j = 0; j < kMaxPerLane; ++j) {
    const int col = lane + 32 * j;
    if (col < columns) {
      dst[col] = __float2half_rn(v[j] * inv_std * __half2float(scale[col]) + __half2float(bias[col]));
    }
  }
}

}  // namespace

extern "C" __global__ void __launch_bounds__(256)
ctb_layer_norm_f16(const __half* x, const __half* scale, const __half* bias, __half* out, int rows,
                   int columns, float epsilon, CTB_RESERVED_PARAMS) {
  CTB_UNUSED_RESERVED();
  CTB_GRID_DEPENDENCY_SYNC();
  const int row = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  if (row >= rows) return;
  const long long offset = static_cast<long long>(row) * columns;
  float v[kMaxPerLane];
  if (vector_rows(x, out, columns) && vector_rows(scale, bias, columns)) {
    load_row_vec(x + offset, columns, v);
    normalize_row_vec(v, columns, epsilon, scale, bias, out + offset);
    return;
  }
  load_row(x + offset, columns, v);
  normalize_row(v, columns, epsilon, scale, bias, out + offset);
}

extern "C" __global__ void __launch_bounds__(256)
ctb_skip_layer_norm_f16(const __half* x, const __half* residual, const __half* scale, const __half* bias,
                        __half* out, int rows, int columns, float epsilon, CTB_RESERVED_PARAMS) {
  CTB_UNUSED_RESERVED();
  CTB_GRID_DEPENDENCY_SYNC();
  const int row = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  if (row >= rows) return;
  const long long offset = static_cast<long long>(row) * columns;
  float v[kMaxPerLane];
  float r[kMaxPerLane];
  if (vector_rows(x, residual, columns) && vector_rows(out, scale, columns) && vector_rows(bias, bias, columns)) {
    load_row_vec(x + offset, columns, v);
    load_row_vec(residual + offset, columns, r);
#pragma unroll
    for (int j = 0; j < kMaxPerLane; ++j) v[j] += r[j];
    normalize_row_vec(v, columns, epsilon, scale, bias, out + offset);
    return;
  }
  load_row(x + offset, columns, v);
  load_row(residual + offset, columns, r);
#pragma unroll
  for (int j = 0; j < kMaxPerLane; ++j) v[j] += r[j];
  normalize_row(v, columns, epsilon, scale, bias, out + offset);
}

extern "C" __global__ void __launch_bounds__(256)
ctb_softmax_f16(const __half* x, __half* out, int rows, int columns, CTB_RESERVED_PARAMS) {
  CTB_UNUSED_RESERVED();
  CTB_GRID_DEPENDENCY_SYNC();
  const int row = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  if (row >= rows) return;
  const int lane = threadIdx.x & 31;
  const long long offset = static_cast<long long>(row) * columns;
  float v[kMaxPerLane];
  float peak = -INFINITY;
#pragma unroll
  for (int j = 0; j < kMaxPerLane; ++j) {
    const int col = lane + 32 * j;
    v[j] = col < columns ? __half2float(x[offset + col]) : -INFINITY;
    peak = fmaxf(peak, v[j]);
  }
  peak = ctb::warp_max(peak);
  float sum = 0.0f;
#pragma unroll
  for (int j = 0; j < kMaxPerLane; ++j) {
    const int col = lane + 32 * j;
    v[j] = col < columns ? expf(v[j] - peak) : 0.0f;
    sum += v[j];
  }
  const float inv = 1.0f / ctb::warp_sum(sum);
#pragma unroll
  for (int j = 0; j < kMaxPerLane; ++j) {
    const int col = lane + 32 * j;
    if (col < columns) out[offset + col] = __float2half_rn(v[j] * inv);
  }
}
