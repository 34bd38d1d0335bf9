// FP32 convolution family and FP32 GEMM on CUDA cores (exact FP32 FMA).
//
// These are the portable variants of the pack: any shape, any stride, pad
// and dilation, and they accumulate every output in the same order as the
// reference kernels (python/cutriton/triton_kernels/resnet.py:12-114 and
// 201-213: one serial sum over k = (c, r, s) per output). The tensor-core
// variants (conv_tc.cu) are the fast path; these keep unusual shapes
// covered and give the tuner a bit-faithful candidate.
//
// Implicit GEMM: rows m = (n, oh, ow) output pixels, columns = output
// channels, k = (ci, r, s). A 64x64 output tile per CTA, k-steps of 16
// staged in shared memory, each of 256 threads owning a 4x4 micro-tile whose
// pixels are 16 apart so that stores of one channel are contiguous.

#include "common.cuh"

namespace {

constexpr int kBM = 64;
constexpr int kBN = 64;
constexpr int kBK = 16;
constexpr int kThreads = 256;

enum Epilogue { kPlain = 0, kBatchNorm = 1, kBatchNormRelu = 2, kBatchNormAddRelu = 3 };

struct ConvShape {
  int n, c, h, w, k, r, s, out_h, out_w, stride_h, stride_w, pad_h, pad_w, dil_h, dil_w;
};

template <int kEpilogue>
__device__ __forceinline__ void conv_simt(const float* __restrict__ x, const float* __restrict__ weight,
                                          const float* __restrict__ scale, const float* __restrict__ bias,
                                          const float* __restrict__ mean, const float* __restrict__ variance,
                                          const float* __restrict__ residual, float* __restrict__ out,
                                          const ConvShape& p, float epsilon) {
  __shared__ float As[kBK][kBM];
  __shared__ float Bs[kBK][kBN + 1];
  const int tid = threadIdx.x;
  const long long pixels_per_image = static_cast<long long>(p.out_h) * p.out_w;
  const long long total_pixels = pixels_per_image * p.n;
  const int kdim = p.c * p.r * p.s;
  const int rs = p.r * p.s;
  const long long m0 = static_cast<long long>(blockIdx.x) * kBM;
  const int n0 = blockIdx.y * kBN;

  // The A-tile element this thread stages: fixed pixel, k rows a_k + 4q.
  const int a_m = tid % kBM;
  const int a_k = tid / kBM;
  const long long a_pixel = m0 + a_m;
  const bool a_valid = a_pixel < total_pixels;
  int ih0 = 0, iw0 = 0;
  long long x_image = 0;
  if (a_valid) {
    const long long img = a_pixel / pixels_per_image;
    const int rem = static_cast<int>(a_pixel % pixels_per_image);
    ih0 = (rem / p.out_w) * p.stride_h - p.pad_h;
    iw0 = (rem % p.out_w) * p.stride_w - p.pad_w;
    x_image = img * p.c * p.h * p.w;
  }
  // The B-tile element: k column b_k, channels b_n + 16q.
  const int b_k = tid % kBK;
  const int b_n = tid / kBK;

  const int tx = tid % 16;  // pixel lane
  const int ty = tid / 16;  // channel lane
  float acc[4][4] = {};

  for (int k0 = 0; k0 < kdim; k0 += kBK) {
#pragma unroll
    for (int q = 0; q < kBK / 4; ++q) {
      const int kk = a_k + 4 * q;
      const int k = k0 + kk;
      float v = 0.0f;
      if (a_valid && k < kdim) {
        const int ci = k / rs;
        const int t = k - ci * rs;
        const int ih = ih0 + (t / p.s) * p.dil_h;
        const int iw = iw0 + (t % p.s) * p.dil_w;
        if (ih >= 0 && ih < p.h && iw >= 0 && iw < p.w) {
          v = __ldg(x + x_image + (static_cast<long long>(ci) * p.h + ih) * p.w + iw);
        }
      }
      As[kk][a_m] = v;
    }
#pragma unroll
    for (int q = 0; q < kBN / 16; ++q) {
      const int nn = b_n + 16 * q;
      const int co = n0 + nn;
      const int k = k0 + b_k;
      Bs[b_k][nn] = (co < p.k && k < kdim) ? __ldg(weight + static_cast<long long>(co) * kdim + k) : 0.0f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < kBK; ++kk) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = As[kk][tx + 16 * i];
#pragma unroll
      for (int j = 0; j < 4; ++j) b[j] = Bs[kk][ty + 16 * j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }

#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int co = n0 + ty + 16 * j;
    if (co >= p.k) continue;
    float mul = 1.0f, m = 0.0f, add = 0.0f;
    if (kEpilogue != kPlain) {
      m = mean[co];
      mul = rsqrtf(variance[co] + epsilon);
      add = bias[co];
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const long long pixel = m0 + tx + 16 * i;
      if (pixel >= total_pixels) continue;
      const long long img = pixel / pixels_per_image;
      const long long rem = pixel % pixels_per_image;
      const long long at = (img * p.k + co) * pixels_per_image + rem;
      float v = acc[i][j];
      if (kEpilogue != kPlain) v = (v - m) * mul * scale[co] + add;
      if (kEpilogue == kBatchNormAddRelu) v += residual[at];
      if (kEpilogue == kBatchNormRelu || kEpilogue == kBatchNormAddRelu) v = fmaxf(v, 0.0f);
      out[at] = v;
    }
  }
}

}  // namespace

#define CTB_CONV_DIMS                                                                           \
  int n, int c, int h, int w, int k, int r, int s, int out_h, int out_w, int stride_h, int stride_w, \
      int pad_h, int pad_w, int dilation_h, int dilation_w
#define CTB_CONV_SHAPE \
  ConvShape{n, c, h, w, k, r, s, out_h, out_w, stride_h, stride_w, pad_h, pad_w, dilation_h, dilation_w}

extern "C" __global__ void __launch_bounds__(kThreads)
ctb_conv_f32_simt(const float* x, const float* weight, float* output, CTB_CONV_DIMS, CTB_RESERVED_PARAMS) {
  CTB_UNUSED_RESERVED();
  CTB_GRID_DEPENDENCY_SYNC();
  conv_simt<kPlain>(x, weight, nullptr, nullptr, nullptr, nullptr, nullptr, output, CTB_CONV_SHAPE, 0.0f);
}

extern "C" __global__ void __launch_bounds__(kThreads)
ctb_conv_bn_f32_simt(const float* x, const float* weight, const float* scale, const float* bias,
                     const float* mean, const float* variance, float* output, CTB_CONV_DIMS, float epsilon,
                     CTB_RESERVED_PARAMS) {
  CTB_UNUSED_RESERVED();
  CTB_GRID_DEPENDENCY_SYNC();
  conv_simt<kBatchNorm>(x, weight, scale, bias, mean, variance, nullptr, output, CTB_CONV_SHAPE, epsilon);
}

extern "C" __global__ void __launch_bounds__(kThreads)
ctb_conv_bn_relu_f32_simt(const float* x, const float* weight, const float* scale, const float* bias,
                          const float* mean, const float* variance, float* output, CTB_CONV_DIMS,
                          float epsilon, CTB_RESERVED_PARAMS) {
  CTB_UNUSED_RESERVED();
  CTB_GRID_DEPENDENCY_SYNC();
  conv_simt<kBatchNormRelu>(x, weight, scale, bias, mean, variance, nullptr, output, CTB_CONV_SHAPE, epsilon);
}

extern "C" __global__ void __launch_bounds__(kThreads)
ctb_conv_bn_add_relu_f32_simt(const float* x, const float* weight, const float* scale, const float* bias,
                              const float* mean, const float* variance, const float* residual, float* output,
                              CTB_CONV_DIMS, float epsilon, CTB_RESERVED_PARAMS) {
  CTB_UNUSED_RESERVED();
  CTB_GRID_DEPENDENCY_SYNC();
  conv_simt<kBatchNormAddRelu>(x, weight, scale, bias, mean, variance, residual, output, CTB_CONV_SHAPE, epsilon);
}

// C[M,N] = A[M,K] . B[K,N], row-major FP32, no bias (resnet.py:201-213).
extern "C" __global__ void __launch_bounds__(kThreads)
ctb_gemm_f32_simt(const float* __restrict__ a, const float* __restrict__ b, float* __restrict__ output, int m,
                  int n, int k, CTB_RESERVED_PARAMS) {
  CTB_UNUSED_RESERVED();
  CTB_GRID_DEPENDENCY_SYNC();
  __shared__ float As[kBK][kBM];
  __shared__ float Bs[kBK][kBN + 1];
  const int tid = threadIdx.x;
  const int m0 = blockIdx.x * kBM;
  const int n0 = blockIdx.y * kBN;
  const int tx = tid % 16;
  const int ty = tid / 16;
  float acc[4][4] = {};
  for (int k0 = 0; k0 < k; k0 += kBK) {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int e = tid + kThreads * q;  // 0..1023 over a 64 x 16 tile
      const int row = e / kBK, kk = e % kBK;
      const int gm = m0 + row, gk = k0 + kk;
      As[kk][row] = (gm < m && gk < k) ? __ldg(a + static_cast<long long>(gm) * k + gk) : 0.0f;
      const int kb = e / kBN, col = e % kBN;
      const int gn = n0 + col, gkb = k0 + kb;
      Bs[kb][col] = (gn < n && gkb < k) ? __ldg(b + static_cast<long long>(gkb) * n + gn) : 0.0f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < kBK; ++kk) {
      float av[4], bv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) av[i] = As[kk][ty + 16 * i];
#pragma unroll
      for (int j = 0; j < 4; ++j) bv[j] = Bs[kk][tx + 16 * j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int gm = m0 + ty + 16 * i;
    if (gm >= m) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int gn = n0 + tx + 16 * j;
      if (gn < n) output[static_cast<long long>(gm) * n + gn] = acc[i][j];
    }
  }
}
