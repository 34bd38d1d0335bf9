// Bandwidth-bound elementwise kernels (FP32 NCHW/contiguous and FP16).
//
// Each CTA of 256 threads owns a contiguous chunk of kChunk elements; every
// thread moves kVecPerThread 16-byte vectors (float4 / 8 halves), all loads
// issued before any store so each thread keeps 4 x 16 B in flight. A chunk
// that is partial, or any operand not 16-byte aligned, takes the scalar path.
// Math follows the reference formulas (python/cutriton/triton_kernels/
// resnet.py:117-156, transformer.py:110-125).

#include "common.cuh"

namespace {

constexpr int kThreads = 256;
constexpr int kVecPerThread = 4;
constexpr int kChunkF32 = kThreads * kVecPerThread * 4;   // 4096 floats
constexpr int kChunkF16 = kThreads * kVecPerThread * 8;   // 8192 halves

struct Relu {
  __device__ float operator()(float a) const { return fmaxf(a, 0.0f); }
};
struct Add {
  __device__ float operator()(float a, float b) const { return a + b; }
};
struct AddRelu {
  __device__ float operator()(float a, float b) const { return fmaxf(a + b, 0.0f); }
};

template <typename Op>
__device__ __forceinline__ void unary_f32(const float* __restrict__ x, float* __restrict__ out, int total, Op op) {
  const long long base = static_cast<long long>(blockIdx.x) * kChunkF32;
  if (base + kChunkF32 <= total && ctb::aligned16(x) && ctb::aligned16(out)) {
    float4 v[kVecPerThread];
#pragma unroll
    for (int j = 0; j < kVecPerThread; ++j) {
      v[j] = reinterpret_cast<const float4*>(x + base)[j * kThreads + threadIdx.x];
    }
#pragma unroll
    for (int j = 0; j < kVecPerThread; ++j) {
      float4 r = make_float4(op(v[j].x), op(v[j].y), op(v[j].z), op(v[j].w));
      reinterpret_cast<float4*>(out + base)[j * kThreads + threadIdx.x] = r;
    }
    return;
  }
  const long long end = min(static_cast<long long>(total), base + kChunkF32);
  for (long long i = base + threadIdx.x; i < end; i += kThreads) out[i] = op(x[i]);
}

template <typename Op>
__device__ __forceinline__ void binary_f32(const float* __restrict__ a, const float* __restrict__ b,
                                           float* __restrict__ out, int total, Op op) {
  const long long base = static_cast<long long>(blockIdx.x) * kChunkF32;
  if (base + kChunkF32 <= total && ctb::aligned16(a) && ctb::aligned16(b) && ctb::aligned16(out)) {
    float4 va[kVecPerThread], vb[kVecPerThread];
#pragma unroll
    for (int j = 0; j < kVecPerThread; ++j) {
      va[j] = reinterpret_cast<const float4*>(a + base)[j * kThreads + threadIdx.x];
      vb[j] = reinterpret_cast<const float4*>(b + base)[j * kThreads + threadIdx.x];
    }
#pragma unroll
    for (int j = 0; j < kVecPerThread; ++j) {
      float4 r = make_float4(op(va[j].x, vb[j].x), op(va[j].y, vb[j].y), op(va[j].z, vb[j].z),
                             op(va[j].w, vb[j].w));
      reinterpret_cast<float4*>(out + base)[j * kThreads + threadIdx.x] = r;
    }
    return;
  }
  const long long end = min(static_cast<long long>(total), base + kChunkF32);
  for (long long i = base + threadIdx.x; i < end; i += kThreads) out[i] = op(a[i], b[i]);
}

}  // namespace

extern "C" __global__ void __launch_bounds__(kThreads)
ctb_relu_f32(const float* x, float* out, int total, CTB_RESERVED_PARAMS) {
  CTB_UNUSED_RESERVED();
  CTB_GRID_DEPENDENCY_SYNC();
  unary_f32(x, out, total, Relu{});
}

extern "C" __global__ void __launch_bounds__(kThreads)
ctb_add_f32(const float* a, const float* b, float* out, int total, CTB_RESERVED_PARAMS) {
  CTB_UNUSED_RESERVED();
  CTB_GRID_DEPENDENCY_SYNC();
  binary_f32(a, b, out, total, Add{});
}

extern "C" __global__ void __launch_bounds__(kThreads)
ctb_add_relu_f32(const float* a, const float* b, float* out, int total, CTB_RESERVED_PARAMS) {
  CTB_UNUSED_RESERVED();
  CTB_GRID_DEPENDENCY_SYNC();
  binary_f32(a, b, out, total, AddRelu{});
}

// Inference BatchNormalization over NCHW: channel = (i / spatial) % channels,
// y = (x - mean) * rsqrt(var + eps) * scale + bias.
extern "C" __global__ void __launch_bounds__(kThreads)
ctb_batch_norm_f32(const float* x, const float* scale, const float* bias, const float* mean,
                   const float* variance, float* out, int total, int channels, int spatial,
                   float epsilon, CTB_RESERVED_PARAMS) {
  CTB_UNUSED_RESERVED();
  CTB_GRID_DEPENDENCY_SYNC();
  auto affine = [&](float v, int c) {
    return (v - mean[c]) * rsqrtf(variance[c] + epsilon) * scale[c] + bias[c];
  };
  const long long base = static_cast<long long>(blockIdx.x) * kChunkF32;
  if (base + kChunkF32 <= total && (spatial & 3) == 0 && ctb::aligned16(x) && ctb::aligned16(out)) {
    float4 v[kVecPerThread];
#pragma unroll
    for (int j = 0; j < kVecPerThread; ++j) {
      v[j] = reinterpret_cast<const float4*>(x + base)[j * kThreads + threadIdx.x];
    }
#pragma unroll
    for (int j = 0; j < kVecPerThread; ++j) {
      const long long i = base + 4LL * (j * kThreads + threadIdx.x);
      const int c = static_cast<int>((i / spatial) % channels);  // 4 | spatial: one channel per vector
      const float4 r = make_float4(affine(v[j].x, c), affine(v[j].y, c), affine(v[j].z, c), affine(v[j].w, c));
      reinterpret_cast<float4*>(out + base)[j * kThreads + threadIdx.x] = r;
    }
    return;
  }
  const long long end = min(static_cast<long long>(total), base + kChunkF32);
  for (long long i = base + threadIdx.x; i < end; i += kThreads) {
    out[i] = affine(x[i], static_cast<int>((i / spatial) % channels));
  }
}

// Exact-erf GELU on FP16 data, computed in FP32, stored round-to-nearest.
extern "C" __global__ void __launch_bounds__(kThreads)
ctb_gelu_f16(const __half* x, __half* out, int total, CTB_RESERVED_PARAMS) {
  CTB_UNUSED_RESERVED();
  CTB_GRID_DEPENDENCY_SYNC();
  const long long base = static_cast<long long>(blockIdx.x) * kChunkF16;
  if (base + kChunkF16 <= total && ctb::aligned16(x) && ctb::aligned16(out)) {
    uint4 v[kVecPerThread];
#pragma unroll
    for (int j = 0; j < kVecPerThread; ++j) v[j] = reinterpret_cast<const uint4*>(x + base)[j * kThreads + threadIdx.x];
#pragma unroll
    for (int j = 0; j < kVecPerThread; ++j) {
      __half2* h = reinterpret_cast<__half2*>(&v[j]);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 f = __half22float2(h[k]);
        h[k] = __floats2half2_rn(ctb::gelu_erf(f.x), ctb::gelu_erf(f.y));
      }
      reinterpret_cast<uint4*>(out + base)[j * kThreads + threadIdx.x] = v[j];
    }
    return;
  }
  const long long end = min(static_cast<long long>(total), base + kChunkF16);
  for (long long i = base + threadIdx.x; i < end; i += kThreads) {
    out[i] = __float2half_rn(ctb::gelu_erf(__half2float(x[i])));
  }
}

// FP16 addition in FP16 arithmetic (the unfused Add of the transformer path).
extern "C" __global__ void __launch_bounds__(kThreads)
ctb_add_f16(const __half* a, const __half* b, __half* out, int total, CTB_RESERVED_PARAMS) {
  CTB_UNUSED_RESERVED();
  CTB_GRID_DEPENDENCY_SYNC();
  const long long base = static_cast<long long>(blockIdx.x) * kChunkF16;
  if (base + kChunkF16 <= total && ctb::aligned16(a) && ctb::aligned16(b) && ctb::aligned16(out)) {
    uint4 va[kVecPerThread], vb[kVecPerThread];
#pragma unroll
    for (int j = 0; j < kVecPerThread; ++j) {
      va[j] = reinterpret_cast<const uint4*>(a + base)[j * kThreads + threadIdx.x];
      vb[j] = reinterpret_cast<const uint4*>(b + base)[j * kThreads + threadIdx.x];
    }
#pragma unroll
    for (int j = 0; j < kVecPerThread; ++j) {
      __half2* ha = reinterpret_cast<__half2*>(&va[j]);
      const __half2* hb = reinterpret_cast<const __half2*>(&vb[j]);
#pragma unroll
      for (int k = 0; k < 4; ++k) ha[k] = __hadd2(ha[k], hb[k]);
      reinterpret_cast<uint4*>(out + base)[j * kThreads + threadIdx.x] = va[j];
    }
    return;
  }
  const long long end = min(static_cast<long long>(total), base + kChunkF16);
  for (long long i = base + threadIdx.x; i < end; i += kThreads) out[i] = __hadd(a[i], b[i]);
}
