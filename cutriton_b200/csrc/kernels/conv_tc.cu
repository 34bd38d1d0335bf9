// FP32 convolution (+BatchNorm [+residual] [+ReLU]) as a 3xTF32 implicit
// GEMM on the 5th-generation tensor cores (tcgen05), NCHW / OIHW.
//
// GEMM view: D[co, pixel] = sum_k W[co, k] * X_im2col[k, pixel], with
// k = (r * S + s) * C + c. FP32 accuracy from TF32 units: each operand is
// split x = hi + lo (hi = x with the low 13 mantissa bits cleared, exactly
// representable in TF32; lo = x - hi) and D accumulates hi*hi + hi*lo + lo*hi
// in FP32 TMEM (the lo*lo term is below FP32 resolution of the sum).
//
// Tile per CTA: 128 output channels (UMMA M) x 128 output pixels (UMMA N),
// k blocks of 32 (one 128-byte swizzle row of FP32), STAGES-deep ring:
//   A (weights) — prepacked once at engine upload to [2][Cout][Kpad]
//       (hi plane, lo plane; "conv_w_tf32x2_okpad"), K-major, loaded by TMA
//       (warp 0 lane 0) into the 128-byte-swizzled canonical layout;
//   B (activations) — gathered by warps 4-7 (one thread per output pixel,
//       im2col addressing with padding/stride/dilation, zero outside the
//       image), split into hi/lo and stored K-major in the same 128-byte
//       swizzle layout as A (one 128-byte row of 32 k values per pixel), then
//       fence.proxy.async + arrive on the stage's full_b barrier;
//   warp 1 lane 0 issues 3 x 4 UMMAs (M128 N128 K8, kind::tf32) per block
//       and commits the stage's empty barrier;
//   warps 0-3 run the epilogue: TMEM lane = output channel, 32 pixels per
//       tcgen05.ld; BN affine (x - mean) * rsqrt(var + eps) * scale + bias
//       (python/cutriton/triton_kernels/resnet.py:41-47), optional residual
//       add and ReLU, FP32 stores.
// All waits are bounded (see tc_common.cuh).

#include "tc_common.cuh"

#ifndef CTB_STAGES
#define CTB_STAGES 3
#endif

namespace {

using namespace ctb::tc;

constexpr int kBM = 128;           // output channels per CTA
constexpr int kBN = 128;           // output pixels per CTA
constexpr int kBK = 32;            // k per block (128 bytes of FP32)
constexpr int kStages = CTB_STAGES;
constexpr int kThreads = 256;
constexpr int kGatherThreads = 128;
constexpr uint32_t kTileA = kBM * kBK * 4;  // 16 KB
constexpr uint32_t kTileB = kBN * kBK * 4;  // 16 KB
constexpr uint32_t kStageBytes = 2 * kTileA + 2 * kTileB;
constexpr uint32_t kTmemCols = kBN;

enum Epilogue { kPlain = 0, kBatchNorm = 1, kBatchNormRelu = 2, kBatchNormAddRelu = 3 };

struct ConvShape {
  int n, c, h, w, k, r, s, out_h, out_w, stride_h, stride_w, pad_h, pad_w, dil_h, dil_w;
};

struct __align__(8) Barriers {
  uint64_t full_a[kStages];
  uint64_t full_b[kStages];
  uint64_t empty[kStages];
  uint64_t accum;
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
  int consumed;
};

// Byte offset of element (k index kk, pixel t) in a K-major 128-byte-swizzled
// B tile: pixel t owns row t (128 bytes = 32 k values); the 16-byte chunks of
// a row are permuted by XOR with (t mod 8), the layout TMA's 128-byte swizzle
// produces and the UMMA descriptor expects.
__device__ __forceinline__ uint32_t b_offset(int kk, int t) {
  return t * 128 + ((((kk >> 2) ^ (t & 7)) & 7) << 4) + (kk & 3) * 4;
}

__device__ __forceinline__ void split_tf32(float x, float* hi, float* lo) {
  const float h = __uint_as_float(__float_as_uint(x) & 0xFFFFE000u);
  *hi = h;
  *lo = x - h;
}

template <int kEpilogue>
__device__ __forceinline__ void conv_tc(const TmaDescriptor* tma_w, const float* __restrict__ x,
                                        const float* __restrict__ scale, const float* __restrict__ bias,
                                        const float* __restrict__ mean, const float* __restrict__ variance,
                                        const float* __restrict__ residual, float* __restrict__ out,
                                        const ConvShape& p, float epsilon, void* scratch) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
  Barriers* bars = reinterpret_cast<Barriers*>(smem + kStages * kStageBytes);
  volatile int* abort = &bars->abort;
  auto a_hi = [&](int s) { return smem + s * kStageBytes; };
  auto a_lo = [&](int s) { return smem + s * kStageBytes + kTileA; };
  auto b_hi = [&](int s) { return smem + s * kStageBytes + 2 * kTileA; };
  auto b_lo = [&](int s) { return smem + s * kStageBytes + 2 * kTileA + kTileB; };

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  const int kdim = p.c * p.r * p.s;
  const int k_blocks = (kdim + kBK - 1) / kBK;
  const long long pixels_per_image = static_cast<long long>(p.out_h) * p.out_w;
  const long long total_pixels = pixels_per_image * p.n;
  const long long pix0 = static_cast<long long>(blockIdx.x) * kBN;
  const int co0 = blockIdx.y * kBM;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bars->full_a[s], 1);
      mbar_init(&bars->full_b[s], kGatherThreads);
      mbar_init(&bars->empty[s], 1);
    }
    mbar_init(&bars->accum, 1);
    mbar_init(&bars->drain, 1);
    bars->abort = 0;
    bars->consumed = 0;
    mbar_init_fence();
    tma_prefetch(tma_w);
  }
  if (warp == 2) tmem_alloc(&bars->tmem_base, kTmemCols);
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  const uint32_t tmem = bars->tmem_base;

  if (warp >= 4) {
    // ---- gather: one thread per output pixel of the tile ----
    const int t = threadIdx.x - 128;
    const long long pixel = pix0 + t;
    const bool valid_pixel = pixel < total_pixels;
    int ih0 = 0, iw0 = 0;
    const float* image = x;
    if (valid_pixel) {
      const long long img = pixel / pixels_per_image;
      const int rem = static_cast<int>(pixel - img * pixels_per_image);
      ih0 = (rem / p.out_w) * p.stride_h - p.pad_h;
      iw0 = (rem % p.out_w) * p.stride_w - p.pad_w;
      image = x + img * p.c * p.h * p.w;
    }
    const long long plane = static_cast<long long>(p.h) * p.w;
    const bool channel_blocks = (p.c % kBK) == 0;
    for (int kb = 0; kb < k_blocks; ++kb) {
      const int s = kb % kStages;
      const int use = kb / kStages;
      if (use > 0 && !mbar_wait(&bars->empty[s], (use - 1) & 1, abort, scratch, 10)) break;
      float v[kBK];
      if (channel_blocks) {
        // One filter tap, 32 consecutive channels.
        const int k0 = kb * kBK;
        const int tap = k0 / p.c;
        const int c0 = k0 - tap * p.c;
        const int ih = ih0 + (tap / p.s) * p.dil_h;
        const int iw = iw0 + (tap % p.s) * p.dil_w;
        const bool inside = valid_pixel && ih >= 0 && ih < p.h && iw >= 0 && iw < p.w;
        const float* src = image + static_cast<long long>(c0) * plane + static_cast<long long>(ih) * p.w + iw;
#pragma unroll
        for (int kk = 0; kk < kBK; ++kk) v[kk] = inside ? __ldg(src + kk * plane) : 0.0f;
      } else {
#pragma unroll 4
        for (int kk = 0; kk < kBK; ++kk) {
          const int k = kb * kBK + kk;
          float value = 0.0f;
          if (valid_pixel && k < kdim) {
            const int tap = k / p.c;
            const int c = k - tap * p.c;
            const int ih = ih0 + (tap / p.s) * p.dil_h;
            const int iw = iw0 + (tap % p.s) * p.dil_w;
            if (ih >= 0 && ih < p.h && iw >= 0 && iw < p.w) {
              value = __ldg(image + static_cast<long long>(c) * plane + static_cast<long long>(ih) * p.w + iw);
            }
          }
          v[kk] = value;
        }
      }
      uint8_t* hi_tile = b_hi(s);
      uint8_t* lo_tile = b_lo(s);
#pragma unroll
      for (int kk = 0; kk < kBK; ++kk) {
        float hi, lo;
        split_tf32(v[kk], &hi, &lo);
        const uint32_t off = b_offset(kk, t);
        *reinterpret_cast<float*>(hi_tile + off) = hi;
        *reinterpret_cast<float*>(lo_tile + off) = lo;
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      mbar_arrive(&bars->full_b[s]);
    }
  } else if (warp == 0 && lane == 0) {
    // ---- TMA producer: weight hi / lo tiles ----
    int issued = 0;
    for (int kb = 0; kb < k_blocks; ++kb) {
      const int s = kb % kStages;
      const int use = kb / kStages;
      if (use > 0 && !mbar_wait(&bars->empty[s], (use - 1) & 1, abort, scratch, 11)) break;
      mbar_arrive_expect_tx(&bars->full_a[s], 2 * kTileA);
      tma_load_3d(a_hi(s), tma_w, &bars->full_a[s], kb * kBK, co0, 0);
      tma_load_3d(a_lo(s), tma_w, &bars->full_a[s], kb * kBK, co0, 1);
      issued = kb + 1;
    }
    if (*abort) {
      for (int kb = *reinterpret_cast<volatile int*>(&bars->consumed); kb < issued; ++kb) {
        volatile int never = 0;
        mbar_wait(&bars->full_a[kb % kStages], (kb / kStages) & 1, &never, scratch, 12);
      }
    }
  } else if (warp == 1 && lane == 0) {
    // ---- UMMA issuer ----
    constexpr uint32_t idesc = instr_desc(kFormatTF32, kBM, kBN);  // A and B K-major
    bool ok = true;
    for (int kb = 0; kb < k_blocks; ++kb) {
      const int s = kb % kStages;
      const uint32_t parity = (kb / kStages) & 1;
      if (!mbar_wait(&bars->full_a[s], parity, abort, scratch, 13) ||
          !mbar_wait(&bars->full_b[s], parity, abort, scratch, 14)) {
        ok = false;
        break;
      }
      tc_fence_after_sync();
      const uint64_t ahi = smem_desc_kmajor_sw128(a_hi(s));
      const uint64_t alo = smem_desc_kmajor_sw128(a_lo(s));
      const uint64_t bhi = smem_desc_kmajor_sw128(b_hi(s));
      const uint64_t blo = smem_desc_kmajor_sw128(b_lo(s));
#pragma unroll
      for (int kk = 0; kk < kBK / 8; ++kk) {
        // +32 bytes (8 TF32 values) along k inside the swizzled rows.
        const uint64_t dk = 2 * kk;
        umma_tf32(tmem, ahi + dk, bhi + dk, idesc, (kb | kk) != 0);
        umma_tf32(tmem, ahi + dk, blo + dk, idesc, 1);
        umma_tf32(tmem, alo + dk, bhi + dk, idesc, 1);
      }
      umma_commit(&bars->empty[s]);
      *reinterpret_cast<volatile int*>(&bars->consumed) = kb + 1;
    }
    umma_commit(ok ? &bars->accum : &bars->drain);
    if (!ok) {
      volatile int never = 0;
      mbar_wait(&bars->drain, 0, &never, scratch, 15);
    }
  }

  if (warp < 4) {
    __syncwarp();
    // ---- epilogue: TMEM lane = output channel, columns = pixels ----
    const bool ready = mbar_wait(&bars->accum, 0, abort, scratch, 16);
    __syncwarp();
    tc_fence_after_sync();
    if (ready) {
      const int co = co0 + warp * 32 + lane;
      const bool valid_co = co < p.k;
      float m = 0.0f, mul = 1.0f, g = 1.0f, b = 0.0f;
      if (kEpilogue != kPlain && valid_co) {
        m = mean[co];
        mul = rsqrtf(variance[co] + epsilon);
        g = scale[co];
        b = bias[co];
      }
      const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;
#pragma unroll 1
      for (int c = 0; c < kBN; c += 32) {
        uint32_t acc[32];
        tmem_load_32x32(tmem + lane_base + c, acc);
        long long pixel = pix0 + c;
        if (!valid_co || pixel >= total_pixels) continue;
        long long img = pixel / pixels_per_image;
        long long rem = pixel - img * pixels_per_image;
        long long at = (img * p.k + co) * pixels_per_image + rem;
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          if (pixel + j < total_pixels) {
            float v = __uint_as_float(acc[j]);
            if (kEpilogue != kPlain) v = (v - m) * mul * g + b;
            if (kEpilogue == kBatchNormAddRelu) v += residual[at];
            if (kEpilogue == kBatchNormRelu || kEpilogue == kBatchNormAddRelu) v = fmaxf(v, 0.0f);
            out[at] = v;
          }
          // Advance to the next pixel (crossing into the next image if needed).
          ++rem;
          ++at;
          if (rem == pixels_per_image) {
            rem = 0;
            ++img;
            at = (img * p.k + co) * pixels_per_image;
          }
        }
      }
    }
  }
  tc_fence_before_sync();
  __syncthreads();
  if (warp == 2) tmem_dealloc(tmem, kTmemCols);
}

}  // namespace

#define CTB_CONV_DIMS                                                                                 \
  int n, int c, int h, int w, int k, int r, int s, int out_h, int out_w, int stride_h, int stride_w, \
      int pad_h, int pad_w, int dilation_h, int dilation_w
#define CTB_CONV_SHAPE \
  ConvShape{n, c, h, w, k, r, s, out_h, out_w, stride_h, stride_w, pad_h, pad_w, dilation_h, dilation_w}

extern "C" __global__ void __launch_bounds__(kThreads, 1)
ctb_conv_f32_tc(const __grid_constant__ TmaDescriptor tma_w, const float* x, float* output, CTB_CONV_DIMS,
                CTB_RESERVED_PARAMS) {
  (void)profile_scratch;
  conv_tc<kPlain>(&tma_w, x, nullptr, nullptr, nullptr, nullptr, nullptr, output, CTB_CONV_SHAPE, 0.0f,
                  runtime_scratch);
}

extern "C" __global__ void __launch_bounds__(kThreads, 1)
ctb_conv_bn_f32_tc(const __grid_constant__ TmaDescriptor tma_w, const float* x, const float* scale,
                   const float* bias, const float* mean, const float* variance, float* output, CTB_CONV_DIMS,
                   float epsilon, CTB_RESERVED_PARAMS) {
  (void)profile_scratch;
  conv_tc<kBatchNorm>(&tma_w, x, scale, bias, mean, variance, nullptr, output, CTB_CONV_SHAPE, epsilon,
                      runtime_scratch);
}

extern "C" __global__ void __launch_bounds__(kThreads, 1)
ctb_conv_bn_relu_f32_tc(const __grid_constant__ TmaDescriptor tma_w, const float* x, const float* scale,
                        const float* bias, const float* mean, const float* variance, float* output,
                        CTB_CONV_DIMS, float epsilon, CTB_RESERVED_PARAMS) {
  (void)profile_scratch;
  conv_tc<kBatchNormRelu>(&tma_w, x, scale, bias, mean, variance, nullptr, output, CTB_CONV_SHAPE, epsilon,
                          runtime_scratch);
}

extern "C" __global__ void __launch_bounds__(kThreads, 1)
ctb_conv_bn_add_relu_f32_tc(const __grid_constant__ TmaDescriptor tma_w, const float* x, const float* scale,
                            const float* bias, const float* mean, const float* variance, const float* residual,
                            float* output, CTB_CONV_DIMS, float epsilon, CTB_RESERVED_PARAMS) {
  (void)profile_scratch;
  conv_tc<kBatchNormAddRelu>(&tma_w, x, scale, bias, mean, variance, residual, output, CTB_CONV_SHAPE, epsilon,
                             runtime_scratch);
}
