// Pooling kernels over NCHW FP32.
//
// MaxPool follows python/cutriton/triton_kernels/resnet.py:159-182: window
// maximum with out-of-range taps contributing -inf, padding taken from
// pads[0] (top) and pads[1] (left). Comparisons are exact, so results are
// bit-identical to any correct implementation. One thread per output; the
// 3x3/2 windows of neighbouring threads overlap, so input rows are served
// from L1 and HBM traffic stays near input + output bytes.
//
// GlobalAveragePool (resnet.py:185-198): the reference sums each plane
// serially, then divides by H*W. Two kernels:
//   * ctb_global_average_pool_f32_staged (planes of at most 81 elements, the
//     7x7 ResNet case): a block copies 128 consecutive planes — one
//     contiguous run of NCHW memory — into shared memory with 16-byte
//     cp.async copies (every thread keeps several in flight), then each
//     thread sums one plane in the reference's order, so results are
//     bit-identical to a serial FP32 loop;
//   * ctb_global_average_pool_f32 (any plane size): one warp per plane,
//     lanes stride the plane, warp-shuffle sum, then the division.

#include <math_constants.h>

#include "common.cuh"

extern "C" __global__ void __launch_bounds__(256)
ctb_max_pool_f32(const float* __restrict__ x, float* __restrict__ out, int n, int c, int h, int w,
                 int out_h, int out_w, int kernel_h, int kernel_w, int stride_h, int stride_w,
                 int pad_h, int pad_w, int dilation_h, int dilation_w, CTB_RESERVED_PARAMS) {
  CTB_UNUSED_RESERVED();
  CTB_GRID_DEPENDENCY_SYNC();
  const long long total = static_cast<long long>(n) * c * out_h * out_w;
  const long long index = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (index >= total) return;
  const int ow = static_cast<int>(index % out_w);
  long long rest = index / out_w;
  const int oh = static_cast<int>(rest % out_h);
  const long long plane = rest / out_h;  // n * c + channel
  const float* src = x + plane * h * w;
  float best = -CUDART_INF_F;
  const int h0 = oh * stride_h - pad_h;
  const int w0 = ow * stride_w - pad_w;
  for (int kh = 0; kh < kernel_h; ++kh) {
    const int ih = h0 + kh * dilation_h;
    if (ih < 0 || ih >= h) continue;
    for (int kw = 0; kw < kernel_w; ++kw) {
      const int iw = w0 + kw * dilation_w;
      if (iw < 0 || iw >= w) continue;
      best = fmaxf(best, __ldg(src + static_cast<long long>(ih) * w + iw));
    }
  }
  out[index] = best;
}

extern "C" __global__ void __launch_bounds__(256)
ctb_global_average_pool_f32(const float* __restrict__ x, float* __restrict__ out, int n, int c, int h,
                            int w, CTB_RESERVED_PARAMS) {
  CTB_UNUSED_RESERVED();
  CTB_GRID_DEPENDENCY_SYNC();
  const int warps_per_block = blockDim.x / 32;
  const long long plane = static_cast<long long>(blockIdx.x) * warps_per_block + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (plane >= static_cast<long long>(n) * c) return;
  const int spatial = h * w;
  const float* src = x + plane * spatial;
  float sum = 0.0f;
  for (int i = lane; i < spatial; i += 32) sum += __ldg(src + i);
  sum = ctb::warp_sum(sum);
  if (lane == 0) out[plane] = sum / static_cast<float>(spatial);
}

// MaxPool 3x3 / stride 2 / pad 1 with W % 4 == 0 and W <= 128 (the ResNet-50
// stem pool): one warp per output row. Lane L loads columns 4L..4L+3 of the
// three input rows as float4 (one 16-byte, fully coalesced access per row)
// and produces outputs 2L (columns 4L-1..4L+1; column 4L-1 is lane L-1's .w,
// passed by a shuffle) and 2L+1 (columns 4L+1..4L+3). Same fmaxf over the
// same taps as ctb_max_pool_f32, so the results are identical.
extern "C" __global__ void __launch_bounds__(256)
ctb_max_pool_3x3s2_f32(const float* __restrict__ x, float* __restrict__ out, int n, int c, int h, int w,
                       int out_h, int out_w, CTB_RESERVED_PARAMS) {
  CTB_UNUSED_RESERVED();
  CTB_GRID_DEPENDENCY_SYNC();
  const long long row = static_cast<long long>(blockIdx.x) * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (row >= static_cast<long long>(n) * c * out_h) return;  // warp-uniform
  const long long plane = row / out_h;
  const int oh = static_cast<int>(row - plane * out_h);
  const float* src = x + plane * h * w;
  const int quads = w / 4;
  const bool vec = (reinterpret_cast<uintptr_t>(x) & 15) == 0;
  float o0 = -CUDART_INF_F, o1 = -CUDART_INF_F;
#pragma unroll
  for (int dr = -1; dr <= 1; ++dr) {
    const int ih = 2 * oh + dr;
    const bool row_ok = ih >= 0 && ih < h;
    float4 v = make_float4(-CUDART_INF_F, -CUDART_INF_F, -CUDART_INF_F, -CUDART_INF_F);
    if (row_ok && lane < quads) {
      const float* p = src + static_cast<long long>(ih) * w + 4 * lane;
      if (vec) {
        v = __ldg(reinterpret_cast<const float4*>(p));
      } else {
        v = make_float4(__ldg(p), __ldg(p + 1), __ldg(p + 2), __ldg(p + 3));
      }
    }
    float left = __shfl_up_sync(0xffffffffu, v.w, 1);
    if (lane == 0) left = -CUDART_INF_F;  // column -1: padding
    o0 = fmaxf(o0, fmaxf(fmaxf(left, v.x), v.y));
    o1 = fmaxf(o1, fmaxf(fmaxf(v.y, v.z), v.w));
  }
  if (lane < quads) {
    float* dst = out + row * out_w + 2 * lane;
    dst[0] = o0;
    dst[1] = o1;
  }
}

// Planes per block and the largest plane the staged kernel takes.
constexpr int kGapPlanes = 128;
constexpr int kGapMaxSpatial = 81;

extern "C" __global__ void __launch_bounds__(kGapPlanes)
ctb_global_average_pool_f32_staged(const float* __restrict__ x, float* __restrict__ out, int n, int c, int h, int w,
                                   CTB_RESERVED_PARAMS) {
  CTB_UNUSED_RESERVED();
  CTB_GRID_DEPENDENCY_SYNC();
  __shared__ __align__(16) float stage[kGapPlanes * kGapMaxSpatial];
  const int spatial = h * w;
  const long long planes = static_cast<long long>(n) * c;
  const long long first = static_cast<long long>(blockIdx.x) * kGapPlanes;
  const int count = static_cast<int>(min(static_cast<long long>(kGapPlanes), planes - first));
  const float* src = x + first * spatial;
  const int elems = count * spatial;
  // 16-byte copies when the run starts on a 16-byte boundary (always for
  // an aligned tensor: first * spatial is a multiple of 128); the ragged
  // end, or a misaligned tensor, goes 4 bytes at a time.
  const bool vector_ok = (reinterpret_cast<uintptr_t>(src) & 15) == 0;
  const int vec = vector_ok ? elems / 4 : 0;
  for (int i = threadIdx.x; i < vec; i += kGapPlanes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(static_cast<uint32_t>(
                     __cvta_generic_to_shared(stage + 4 * i))),
                 "l"(src + 4 * i)
                 : "memory");
  }
  for (int i = 4 * vec + threadIdx.x; i < elems; i += kGapPlanes) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(static_cast<uint32_t>(
                     __cvta_generic_to_shared(stage + i))),
                 "l"(src + i)
                 : "memory");
  }
  asm volatile("cp.async.wait_all;" ::: "memory");
  __syncthreads();
  if (threadIdx.x < count) {
    // Row stride `spatial` (odd for 7x7): consecutive threads hit distinct banks.
    const float* plane = stage + threadIdx.x * spatial;
    float sum = 0.0f;
    for (int i = 0; i < spatial; ++i) sum += plane[i];
    out[first + threadIdx.x] = sum / static_cast<float>(spatial);
  }
}
