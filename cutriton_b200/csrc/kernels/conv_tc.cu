// FP32 convolution (+BatchNorm [+residual] [+ReLU]) as a 3xTF32 implicit
// GEMM on the 5th-generation tensor cores (tcgen05), NCHW / OIHW.
//
// GEMM view: D[co, pixel] = sum_k W[co, k] * X_im2col[k, pixel] with
// k = (r * S + s) * Cp + c (Cp = C when C % 32 == 0, else C rounded up to a
// multiple of 4; padded channels carry zero weights). FP32 accuracy from
// TF32 units: each operand is split x = hi + lo (hi = x with the low 13
// mantissa bits cleared, exactly representable in TF32; lo = x - hi) and D
// accumulates hi*hi + hi*lo + lo*hi in FP32 TMEM.
//
// Persistent kernel: one CTA per SM walks the output tiles (128 output
// channels x 128 output pixels) in a static round-robin. Roles (10 warps):
//   warp 0 lane 0 — TMA producer of the weight tiles: prepacked at engine
//       upload to [2][Cout][Kpad] (hi plane, lo plane; "conv_w_tf32x2_okpad"),
//       K-major, 128-byte swizzle, k blocks of 32 through a STAGES ring;
//   warps 6-9 — gather, one thread per output pixel: im2col addressing with
//       padding/stride/dilation (zero outside the image), the next block's
//       global loads issued before the current block is stored; hi/lo split
//       written K-major as 16-byte swizzled chunks, then fence.proxy.async +
//       arrive on the stage's full_b barrier;
//   warp 1 lane 0 — UMMA issuer: 3 x 4 UMMAs (M128 N128 K8, kind::tf32) per
//       block into one of two TMEM accumulators (2 x 128 columns), commit of
//       the stage's empty barrier per block and of the accumulator's full
//       barrier per tile;
//   warps 2-5 — epilogue of the previous tile while the next one computes:
//       TMEM lane quarter (warp % 4) = 32 output channels; BN affine
//       (x - mean) * rsqrt(var + eps) * scale + bias (python/cutriton/
//       triton_kernels/resnet.py:41-47) per channel, a 32x32 transpose through
//       shared memory so each warp store covers 32 consecutive pixels of one
//       channel (128 contiguous bytes), optional residual add and ReLU; then
//       the accumulator is handed back to the issuer.
// All waits are bounded (see tc_common.cuh).

#include "tc_common.cuh"

#ifndef CTB_STAGES
#define CTB_STAGES 3
#endif

namespace {

using namespace ctb::tc;

constexpr int kBM = 128;           // output channels per tile
constexpr int kBN = 128;           // output pixels per tile
constexpr int kBK = 32;            // k per block (128 bytes of FP32)
constexpr int kStages = CTB_STAGES;
constexpr int kThreads = 320;
constexpr int kEpilogueWarp0 = 2;
constexpr int kGatherWarp0 = 6;
constexpr int kGatherThreads = 128;
constexpr uint32_t kTileA = kBM * kBK * 4;  // 16 KB
constexpr uint32_t kTileB = kBN * kBK * 4;  // 16 KB
constexpr uint32_t kStageBytes = 2 * kTileA + 2 * kTileB;
constexpr int kStagePitch = 33;             // transpose buffer row pitch (floats)
constexpr uint32_t kEpilogueBytes = 4 * 32 * kStagePitch * 4;
constexpr uint32_t kTmemCols = 2 * kBN;     // two accumulators

enum Epilogue { kPlain = 0, kBatchNorm = 1, kBatchNormRelu = 2, kBatchNormAddRelu = 3 };

struct ConvShape {
  int n, c, h, w, k, r, s, out_h, out_w, stride_h, stride_w, pad_h, pad_w, dil_h, dil_w;
};

struct __align__(8) Barriers {
  uint64_t full_a[kStages];
  uint64_t full_b[kStages];
  uint64_t empty[kStages];
  uint64_t tmem_full[2];
  uint64_t tmem_empty[2];
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
  int consumed;
};

__device__ __forceinline__ float tf32_hi(float x) { return __uint_as_float(__float_as_uint(x) & 0xFFFFE000u); }

struct PixelSource {
  const float* image;
  int ih0, iw0;
  bool valid;
};

// Loads the 32 k values of block `kb` for one pixel (im2col, zero padding).
__device__ __forceinline__ void gather_block(const PixelSource& px, const ConvShape& p, int cp, int kdim,
                                             long long plane, int kb, float (&v)[kBK]) {
  if (p.c % kBK == 0) {
    // One filter tap, 32 consecutive channels.
    const int k0 = kb * kBK;
    const int tap = k0 / cp;
    const int c0 = k0 - tap * cp;
    const int r = tap / p.s;
    const int ih = px.ih0 + r * p.dil_h;
    const int iw = px.iw0 + (tap - r * p.s) * p.dil_w;
    const bool inside = px.valid && ih >= 0 && ih < p.h && iw >= 0 && iw < p.w;
    const float* src = px.image + static_cast<long long>(c0) * plane + static_cast<long long>(ih) * p.w + iw;
#pragma unroll
    for (int kk = 0; kk < kBK; ++kk) v[kk] = inside ? __ldg(src + kk * plane) : 0.0f;
  } else {
    // Chunks of 4 k: four channels of one tap (cp is a multiple of 4).
#pragma unroll
    for (int j = 0; j < kBK / 4; ++j) {
      const int k = kb * kBK + 4 * j;
      const int tap = k / cp;
      const int c = k - tap * cp;
      const int r = tap / p.s;
      const int ih = px.ih0 + r * p.dil_h;
      const int iw = px.iw0 + (tap - r * p.s) * p.dil_w;
      const bool inside = px.valid && k < kdim && ih >= 0 && ih < p.h && iw >= 0 && iw < p.w;
      const float* src = px.image + static_cast<long long>(c) * plane + static_cast<long long>(ih) * p.w + iw;
#pragma unroll
      for (int i = 0; i < 4; ++i) v[4 * j + i] = (inside && c + i < p.c) ? __ldg(src + i * plane) : 0.0f;
    }
  }
}

// Writes one pixel's 32 k values as hi / lo rows of the K-major swizzled
// tiles: row t (128 bytes), 16-byte chunk j stored at chunk j ^ (t mod 8).
__device__ __forceinline__ void store_block(uint8_t* hi_tile, uint8_t* lo_tile, int t, const float (&v)[kBK]) {
#pragma unroll
  for (int j = 0; j < kBK / 4; ++j) {
    const uint32_t off = t * 128 + (((j ^ t) & 7) << 4);
    float4 h, l;
    h.x = tf32_hi(v[4 * j + 0]);
    h.y = tf32_hi(v[4 * j + 1]);
    h.z = tf32_hi(v[4 * j + 2]);
    h.w = tf32_hi(v[4 * j + 3]);
    l.x = v[4 * j + 0] - h.x;
    l.y = v[4 * j + 1] - h.y;
    l.z = v[4 * j + 2] - h.z;
    l.w = v[4 * j + 3] - h.w;
    *reinterpret_cast<float4*>(hi_tile + off) = h;
    *reinterpret_cast<float4*>(lo_tile + off) = l;
  }
}

template <int kEpilogue>
__device__ __forceinline__ void conv_tc(const TmaDescriptor* tma_w, const float* __restrict__ x,
                                        const float* __restrict__ scale, const float* __restrict__ bias,
                                        const float* __restrict__ mean, const float* __restrict__ variance,
                                        const float* __restrict__ residual, float* __restrict__ out,
                                        const ConvShape& p, float epsilon, void* scratch) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
  float* epilogue_smem = reinterpret_cast<float*>(smem + kStages * kStageBytes);
  Barriers* bars = reinterpret_cast<Barriers*>(smem + kStages * kStageBytes + kEpilogueBytes);
  volatile int* abort = &bars->abort;
  auto a_hi = [&](int s) { return smem + s * kStageBytes; };
  auto a_lo = [&](int s) { return smem + s * kStageBytes + kTileA; };
  auto b_hi = [&](int s) { return smem + s * kStageBytes + 2 * kTileA; };
  auto b_lo = [&](int s) { return smem + s * kStageBytes + 2 * kTileA + kTileB; };

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  const int cp = p.c % kBK == 0 ? p.c : (p.c + 3) & ~3;
  const int kdim = cp * p.r * p.s;
  const int k_blocks = (kdim + kBK - 1) / kBK;
  const long long pixels_per_image = static_cast<long long>(p.out_h) * p.out_w;
  const long long total_pixels = pixels_per_image * p.n;
  const int co_tiles = (p.k + kBM - 1) / kBM;
  const long long tiles = ((total_pixels + kBN - 1) / kBN) * co_tiles;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bars->full_a[s], 1);
      mbar_init(&bars->full_b[s], kGatherThreads);
      mbar_init(&bars->empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&bars->tmem_full[b], 1);
      mbar_init(&bars->tmem_empty[b], 4);
    }
    mbar_init(&bars->drain, 1);
    bars->abort = 0;
    bars->consumed = 0;
    mbar_init_fence();
    tma_prefetch(tma_w);
  }
  if (warp == 0) tmem_alloc(&bars->tmem_base, kTmemCols);
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  const uint32_t tmem = bars->tmem_base;
  // Activations are touched only after the preceding kernel has finished.
  CTB_GRID_DEPENDENCY_SYNC();

  if (warp >= kGatherWarp0) {
    // ---- gather: one thread per output pixel of the tile ----
    const int t = threadIdx.x - kGatherWarp0 * 32;
    const long long plane = static_cast<long long>(p.h) * p.w;
    long long g = 0;  // global k-block counter (stage ring position)
    bool stop = false;
    for (long long tile = blockIdx.x; tile < tiles && !stop; tile += gridDim.x) {
      const long long pixel = (tile / co_tiles) * kBN + t;
      PixelSource px{x, 0, 0, pixel < total_pixels};
      if (px.valid) {
        const long long img = pixel / pixels_per_image;
        const int rem = static_cast<int>(pixel - img * pixels_per_image);
        px.ih0 = (rem / p.out_w) * p.stride_h - p.pad_h;
        px.iw0 = (rem % p.out_w) * p.stride_w - p.pad_w;
        px.image = x + img * p.c * p.h * p.w;
      }
      float cur[kBK], nxt[kBK];
      gather_block(px, p, cp, kdim, plane, 0, cur);
      for (int kb = 0; kb < k_blocks; ++kb, ++g) {
        const int s = static_cast<int>(g % kStages);
        const long long use = g / kStages;
        if (kb + 1 < k_blocks) gather_block(px, p, cp, kdim, plane, kb + 1, nxt);
        if (use > 0 && !mbar_wait(&bars->empty[s], (use - 1) & 1, abort, scratch, 10)) {
          stop = true;
          break;
        }
        store_block(b_hi(s), b_lo(s), t, cur);
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        mbar_arrive(&bars->full_b[s]);
#pragma unroll
        for (int kk = 0; kk < kBK; ++kk) cur[kk] = nxt[kk];
      }
    }
  } else if (warp == 0 && lane == 0) {
    // ---- TMA producer: weight hi / lo tiles ----
    long long g = 0;
    bool stop = false;
    for (long long tile = blockIdx.x; tile < tiles && !stop; tile += gridDim.x) {
      const int co0 = static_cast<int>(tile % co_tiles) * kBM;
      for (int kb = 0; kb < k_blocks; ++kb, ++g) {
        const int s = static_cast<int>(g % kStages);
        const long long use = g / kStages;
        if (use > 0 && !mbar_wait(&bars->empty[s], (use - 1) & 1, abort, scratch, 11)) {
          stop = true;
          break;
        }
        mbar_arrive_expect_tx(&bars->full_a[s], 2 * kTileA);
        tma_load_3d(a_hi(s), tma_w, &bars->full_a[s], kb * kBK, co0, 0);
        tma_load_3d(a_lo(s), tma_w, &bars->full_a[s], kb * kBK, co0, 1);
      }
    }
    if (*abort) {
      // Let every issued copy land before the CTA's shared memory is released.
      const long long issued = g;
      for (long long q = *reinterpret_cast<volatile int*>(&bars->consumed); q < issued; ++q) {
        volatile int never = 0;
        mbar_wait(&bars->full_a[q % kStages], (q / kStages) & 1, &never, scratch, 12);
      }
    }
  } else if (warp == 1 && lane == 0) {
    // ---- UMMA issuer ----
    constexpr uint32_t idesc = instr_desc(kFormatTF32, kBM, kBN);  // A and B K-major
    long long g = 0;
    int local = 0;
    bool ok = true;
    for (long long tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x, ++local) {
      const int buf = local & 1;
      if (local >= 2 && !mbar_wait(&bars->tmem_empty[buf], ((local >> 1) - 1) & 1, abort, scratch, 17)) {
        ok = false;
        break;
      }
      tc_fence_after_sync();
      const uint32_t acc = tmem + buf * kBN;
      for (int kb = 0; kb < k_blocks; ++kb, ++g) {
        const int s = static_cast<int>(g % kStages);
        const uint32_t parity = (g / kStages) & 1;
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
          umma_tf32(acc, ahi + dk, bhi + dk, idesc, (kb | kk) != 0);
          umma_tf32(acc, ahi + dk, blo + dk, idesc, 1);
          umma_tf32(acc, alo + dk, bhi + dk, idesc, 1);
        }
        umma_commit(&bars->empty[s]);
        *reinterpret_cast<volatile int*>(&bars->consumed) = static_cast<int>(g + 1);
      }
      if (ok) umma_commit(&bars->tmem_full[buf]);
    }
    if (!ok) {
      umma_commit(&bars->drain);
      volatile int never = 0;
      mbar_wait(&bars->drain, 0, &never, scratch, 15);
    }
  } else if (warp >= kEpilogueWarp0 && warp < kEpilogueWarp0 + 4) {
    // ---- epilogue ----
    const int quarter = warp & 3;  // TMEM lanes this warp may access
    float* stage = epilogue_smem + (warp - kEpilogueWarp0) * 32 * kStagePitch;
    const long long channel_stride = pixels_per_image;
    int local = 0;
    for (long long tile = blockIdx.x; tile < tiles; tile += gridDim.x, ++local) {
      const int buf = local & 1;
      const bool ready = mbar_wait(&bars->tmem_full[buf], (local >> 1) & 1, abort, scratch, 16);
      __syncwarp();
      if (!ready) break;
      tc_fence_after_sync();
      const long long pix0 = (tile / co_tiles) * kBN;
      const int co_base = static_cast<int>(tile % co_tiles) * kBM + quarter * 32;
      const int my_co = co_base + lane;
      float m = 0.0f, mul = 1.0f, g = 1.0f, b = 0.0f;
      if (kEpilogue != kPlain && my_co < p.k) {
        m = mean[my_co];
        mul = rsqrtf(variance[my_co] + epsilon);
        g = scale[my_co];
        b = bias[my_co];
      }
      const uint32_t taddr = tmem + buf * kBN + (static_cast<uint32_t>(quarter * 32) << 16);
      const int rows = min(32, p.k - co_base);
#pragma unroll 1
      for (int c = 0; c < kBN; c += 32) {
        uint32_t accv[32];
        tmem_load_32x32(taddr + c, accv);
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          float v = __uint_as_float(accv[j]);
          if (kEpilogue != kPlain) v = (v - m) * mul * g + b;
          stage[lane * kStagePitch + j] = v;
        }
        __syncwarp();
        // Lane = pixel now: stores of one channel are 128 contiguous bytes.
        const long long pixel = pix0 + c + lane;
        if (pixel < total_pixels && rows > 0) {
          const long long img = pixel / pixels_per_image;
          const long long base = img * p.k * channel_stride + (pixel - img * pixels_per_image);
          float res[32];
          if (kEpilogue == kBatchNormAddRelu) {
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              res[i] = i < rows ? __ldg(residual + base + static_cast<long long>(co_base + i) * channel_stride)
                                : 0.0f;
            }
          }
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            if (i < rows) {
              const long long at = base + static_cast<long long>(co_base + i) * channel_stride;
              float v = stage[i * kStagePitch + lane];
              if (kEpilogue == kBatchNormAddRelu) v += res[i];
              if (kEpilogue == kBatchNormRelu || kEpilogue == kBatchNormAddRelu) v = fmaxf(v, 0.0f);
              out[at] = v;
            }
          }
        }
        __syncwarp();
      }
      // Hand the accumulator back to the issuer.
      tc_fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->tmem_empty[buf]);
    }
  }
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  if (warp == 0) {
    __syncwarp();
    tmem_dealloc(tmem, kTmemCols);
  }
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
