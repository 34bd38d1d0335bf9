// FP32 convolution (+BatchNorm [+residual] [+ReLU]) as a 3xTF32 implicit
// GEMM on the 5th-generation tensor cores with the activation operand held in
// tensor memory (TMEM), NCHW / OIHW.
//
// GEMM view: D[pixel, co] = sum_k X_im2col[pixel, k] * W[co, k] with
// k = (r * S + s) * Cp + c (Cp = C when C % 32 == 0, else C rounded up to a
// multiple of 4; padded channels carry zero weights). FP32 accuracy from TF32
// units: each operand is split x = hi + lo (hi = x with the low 13 mantissa
// bits cleared, exact in TF32; lo = x - hi) and D accumulates
// hi*hi + hi*lo + lo*hi in FP32.
//
// Why the activations live in TMEM: with both operands in shared memory a
// 128x128 UMMA reads 8 KB of shared memory per 64 tensor-core clocks, and the
// three products per k block plus the operand writes need ~200 B/clk — above
// the 128 B/clk an SM's shared memory delivers. With A in TMEM the UMMAs read
// only the weight tile from shared memory (64 B/clk) and the activations go
// register -> TMEM without touching shared memory. It also makes both global
// access patterns natural for NCHW: TMEM lane = output pixel, so a warp's 32
// lanes read (gather) and write (epilogue) 32 consecutive pixels of one
// channel — 128 contiguous bytes per instruction, no transpose.
//
// Persistent kernel: one CTA per SM walks the tiles (128 output pixels x BN
// output channels, BN = 64 when Cout <= 64 else 128) in a static round-robin,
// channel tile fastest so CTAs running together share activations in L2.
// TMEM (512 columns): two BN-column accumulators, then STAGES activation
// stages of 64 columns (32 hi + 32 lo). Roles (14 warps):
//   warp 0 lane 0 — TMA producer of the weight tiles, prepacked at engine
//       upload to [2][Cout][Kpad] (hi plane, lo plane; "conv_w_tf32x2_okpad"),
//       K-major, 128-byte swizzle, boxes of 32 k x 64 channels;
//   warps 6-13 — gather in two groups of four warps (one per TMEM lane
//       quarter) taking alternate k blocks: one thread per output pixel, im2col
//       addressing with padding/stride/dilation (zero outside the image), the
//       group's next block loaded before the current one is stored; hi/lo split
//       written with tcgen05.st, then wait::st + fence + arrive on full_a;
//   warp 1 lane 0 — UMMA issuer: 3 x 4 UMMAs (M128 N=BN K8, kind::tf32, A from
//       TMEM, B from shared memory) per k block, commit of the stage's empty
//       barrier per block and of the accumulator's full barrier per tile;
//   warps 2-5 — epilogue of the previous tile while the next one computes:
//       lane = pixel, 32 channels per TMEM load; BN affine
//       (x - mean) * rsqrt(var + eps) * scale + bias (python/cutriton/
//       triton_kernels/resnet.py:41-47), optional residual add and ReLU, stores
//       of 32 consecutive pixels per channel.
// All waits are bounded (see tc_common.cuh).

#include "tc_common.cuh"

namespace {

using namespace ctb::tc;

constexpr int kBM = 128;  // output pixels per tile (TMEM lanes)
constexpr int kBK = 32;   // k per block (128 bytes of FP32)
constexpr int kThreads = 448;
constexpr int kEpilogueWarp0 = 2;
constexpr int kGatherWarp0 = 6;
constexpr int kGroupThreads = 128;    // four warps, one per lane quarter
constexpr int kBoxRows = 64;          // weight rows (output channels) per TMA box
constexpr uint32_t kBoxBytes = kBoxRows * kBK * 4;  // 8 KB
constexpr uint32_t kTmemCols = 512;
constexpr int kMaxStages = 6;
constexpr uint32_t kStageRegionBytes = 131072;      // max over configurations
constexpr uint32_t kParamBytes = 4 * 32 * 4 * 3;    // per epilogue warp: mean, scale, bias x 32

template <int BN>
struct Tile {
  static constexpr int kStages = BN == 64 ? 6 : 4;
  static constexpr uint32_t kPlaneBytes = BN * kBK * 4;  // one of hi / lo
  static constexpr uint32_t kStageBytes = 2 * kPlaneBytes;
  static constexpr uint32_t kAColumn0 = 2 * BN;          // first activation stage column
  static_assert(kAColumn0 + kStages * 2 * kBK <= kTmemCols, "TMEM budget");
  static_assert(kStages * kStageBytes <= kStageRegionBytes, "shared memory budget");
};

enum Epilogue { kPlain = 0, kBatchNorm = 1, kBatchNormRelu = 2, kBatchNormAddRelu = 3 };

struct ConvShape {
  int n, c, h, w, k, r, s, out_h, out_w, stride_h, stride_w, pad_h, pad_w, dil_h, dil_w;
};

struct __align__(8) Barriers {
  uint64_t full_a[kMaxStages];
  uint64_t full_b[kMaxStages];
  uint64_t empty[kMaxStages];
  uint64_t tmem_full[2];
  uint64_t tmem_empty[2];
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
  int consumed;
};

// 32 lanes x 32 consecutive 32-bit columns from registers: thread t of the
// warp writes row (lane base + t).
__device__ __forceinline__ void tmem_store_32x32(uint32_t taddr, const uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
      "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]),
      "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]),
      "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]),
      "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
      : "memory");
}

__device__ __forceinline__ void tmem_store_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// D[tmem] (+)= A[tmem] . B[smem]^T, TF32 inputs.
__device__ __forceinline__ void umma_tf32_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n\t}"
      ::"r"(d_tmem), "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

struct PixelSource {
  const float* image;
  int ih0, iw0;
  bool valid;
};

__device__ __forceinline__ PixelSource pixel_source(const float* x, const ConvShape& p, long long pixel,
                                                    long long total_pixels, long long pixels_per_image) {
  PixelSource px{x, 0, 0, pixel < total_pixels};
  if (px.valid) {
    const long long img = pixel / pixels_per_image;
    const int rem = static_cast<int>(pixel - img * pixels_per_image);
    const int oh = rem / p.out_w;
    px.ih0 = oh * p.stride_h - p.pad_h;
    px.iw0 = (rem - oh * p.out_w) * p.stride_w - p.pad_w;
    px.image = x + img * p.c * static_cast<long long>(p.h) * p.w;
  }
  return px;
}

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

template <int kEpilogue, int BN>
__device__ __forceinline__ void conv_tm(uint8_t* smem, const TmaDescriptor* tma_w, const float* __restrict__ x,
                                        const float* __restrict__ scale, const float* __restrict__ bias,
                                        const float* __restrict__ mean, const float* __restrict__ variance,
                                        const float* __restrict__ residual, float* __restrict__ out,
                                        const ConvShape& p, float epsilon, void* scratch) {
  using T = Tile<BN>;
  constexpr int kStages = T::kStages;
  float* params = reinterpret_cast<float*>(smem + kStageRegionBytes);
  Barriers* bars = reinterpret_cast<Barriers*>(smem + kStageRegionBytes + kParamBytes);
  volatile int* abort = &bars->abort;
  auto b_hi = [&](int s) { return smem + s * T::kStageBytes; };
  auto b_lo = [&](int s) { return smem + s * T::kStageBytes + T::kPlaneBytes; };

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  const int cp = p.c % kBK == 0 ? p.c : (p.c + 3) & ~3;
  const int kdim = cp * p.r * p.s;
  const int k_blocks = (kdim + kBK - 1) / kBK;
  const long long pixels_per_image = static_cast<long long>(p.out_h) * p.out_w;
  const long long total_pixels = pixels_per_image * p.n;
  const int co_tiles = (p.k + BN - 1) / BN;
  const long long tiles = ((total_pixels + kBM - 1) / kBM) * co_tiles;
  const int my_tiles = tiles > blockIdx.x ? static_cast<int>((tiles - 1 - blockIdx.x) / gridDim.x) + 1 : 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bars->full_a[s], kGroupThreads);
      mbar_init(&bars->full_b[s], 1);
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

  if (warp >= kGatherWarp0) {
    // ---- gather: one thread per output pixel, alternate k blocks per group ----
    const int group = (warp - kGatherWarp0) / 4;
    const int row = (warp & 3) * 32 + lane;  // TMEM lane = pixel within the tile
    const uint32_t lane_bits = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const long long plane = static_cast<long long>(p.h) * p.w;
    const int items = my_tiles * k_blocks;  // this CTA's k blocks, in issue order
    auto fetch = [&](int item, float (&v)[kBK]) {
      const int local = item / k_blocks;
      const int kb = item - local * k_blocks;
      const long long tile = blockIdx.x + static_cast<long long>(local) * gridDim.x;
      const PixelSource px =
          pixel_source(x, p, (tile / co_tiles) * kBM + row, total_pixels, pixels_per_image);
      gather_block(px, p, cp, kdim, plane, kb, v);
    };
    float cur[kBK], nxt[kBK];
    int item = group;
    if (item < items) fetch(item, cur);
    for (; item < items; item += 2) {
      if (item + 2 < items) fetch(item + 2, nxt);
      const int s = item % kStages;
      const int use = item / kStages;
      if (use > 0 && !mbar_wait(&bars->empty[s], (use - 1) & 1, abort, scratch, 30)) break;
      tc_fence_after_sync();
      const uint32_t a_col = tmem + lane_bits + T::kAColumn0 + s * 2 * kBK;
      uint32_t hi[kBK], lo[kBK];
#pragma unroll
      for (int kk = 0; kk < kBK; ++kk) {
        hi[kk] = __float_as_uint(cur[kk]) & 0xFFFFE000u;
        lo[kk] = __float_as_uint(cur[kk] - __uint_as_float(hi[kk]));
      }
      tmem_store_32x32(a_col, hi);
      tmem_store_32x32(a_col + kBK, lo);
      tmem_store_wait();
      tc_fence_before_sync();
      mbar_arrive(&bars->full_a[s]);
#pragma unroll
      for (int kk = 0; kk < kBK; ++kk) cur[kk] = nxt[kk];
    }
  } else if (warp == 0 && lane == 0) {
    // ---- TMA producer: weight hi / lo tiles ----
    int g = 0;
    bool stop = false;
    for (int local = 0; local < my_tiles && !stop; ++local) {
      const long long tile = blockIdx.x + static_cast<long long>(local) * gridDim.x;
      const int co0 = static_cast<int>(tile % co_tiles) * BN;
      for (int kb = 0; kb < k_blocks; ++kb, ++g) {
        const int s = g % kStages;
        const int use = g / kStages;
        if (use > 0 && !mbar_wait(&bars->empty[s], (use - 1) & 1, abort, scratch, 31)) {
          stop = true;
          break;
        }
        mbar_arrive_expect_tx(&bars->full_b[s], 2 * T::kPlaneBytes);
#pragma unroll
        for (int b = 0; b < BN / kBoxRows; ++b) {
          tma_load_3d(b_hi(s) + b * kBoxBytes, tma_w, &bars->full_b[s], kb * kBK, co0 + b * kBoxRows, 0);
          tma_load_3d(b_lo(s) + b * kBoxBytes, tma_w, &bars->full_b[s], kb * kBK, co0 + b * kBoxRows, 1);
        }
      }
    }
    if (*abort) {
      // Let every issued copy land before the CTA's shared memory is released.
      for (int q = *reinterpret_cast<volatile int*>(&bars->consumed); q < g; ++q) {
        volatile int never = 0;
        mbar_wait(&bars->full_b[q % kStages], (q / kStages) & 1, &never, scratch, 32);
      }
    }
  } else if (warp == 1 && lane == 0) {
    // ---- UMMA issuer ----
    constexpr uint32_t idesc = instr_desc(kFormatTF32, kBM, BN);  // A (TMEM) and B K-major
    int g = 0;
    bool ok = true;
    for (int local = 0; local < my_tiles && ok; ++local) {
      const int buf = local & 1;
      if (local >= 2 && !mbar_wait(&bars->tmem_empty[buf], ((local >> 1) - 1) & 1, abort, scratch, 33)) {
        ok = false;
        break;
      }
      tc_fence_after_sync();
      const uint32_t acc = tmem + buf * BN;
      for (int kb = 0; kb < k_blocks; ++kb, ++g) {
        const int s = g % kStages;
        const uint32_t parity = (g / kStages) & 1;
        if (!mbar_wait(&bars->full_b[s], parity, abort, scratch, 34) ||
            !mbar_wait(&bars->full_a[s], parity, abort, scratch, 35)) {
          ok = false;
          break;
        }
        tc_fence_after_sync();
        const uint64_t bhi = smem_desc_kmajor_sw128(b_hi(s));
        const uint64_t blo = smem_desc_kmajor_sw128(b_lo(s));
        const uint32_t ahi = tmem + T::kAColumn0 + s * 2 * kBK;
        const uint32_t alo = ahi + kBK;
#pragma unroll
        for (int kk = 0; kk < kBK / 8; ++kk) {
          // 8 TF32 values along k: 8 TMEM columns of A, +32 bytes inside B's rows.
          const uint64_t dk = 2 * kk;
          umma_tf32_ts(acc, ahi + 8 * kk, bhi + dk, idesc, (kb | kk) != 0);
          umma_tf32_ts(acc, ahi + 8 * kk, blo + dk, idesc, 1);
          umma_tf32_ts(acc, alo + 8 * kk, bhi + dk, idesc, 1);
        }
        umma_commit(&bars->empty[s]);
        *reinterpret_cast<volatile int*>(&bars->consumed) = g + 1;
      }
      if (ok) umma_commit(&bars->tmem_full[buf]);
    }
    if (!ok) {
      umma_commit(&bars->drain);
      volatile int never = 0;
      mbar_wait(&bars->drain, 0, &never, scratch, 36);
    }
  } else if (warp >= kEpilogueWarp0 && warp < kEpilogueWarp0 + 4) {
    // ---- epilogue: lane = output pixel, 32 channels per TMEM load ----
    const int quarter = warp & 3;  // TMEM lanes this warp may access
    float* prm = params + (warp - kEpilogueWarp0) * 32 * 3;
    for (int local = 0; local < my_tiles; ++local) {
      const int buf = local & 1;
      const bool ready = mbar_wait(&bars->tmem_full[buf], (local >> 1) & 1, abort, scratch, 37);
      __syncwarp();
      if (!ready) break;
      tc_fence_after_sync();
      const long long tile = blockIdx.x + static_cast<long long>(local) * gridDim.x;
      const int co0 = static_cast<int>(tile % co_tiles) * BN;
      const long long pixel = (tile / co_tiles) * kBM + quarter * 32 + lane;
      const bool valid = pixel < total_pixels;
      long long base = 0;  // output offset of (image, channel 0, pixel)
      if (valid) {
        const long long img = pixel / pixels_per_image;
        base = img * p.k * pixels_per_image + (pixel - img * pixels_per_image);
      }
      const uint32_t taddr = tmem + buf * BN + (static_cast<uint32_t>(quarter * 32) << 16);
#pragma unroll 1
      for (int c = 0; c < BN; c += 32) {
        const int ch0 = co0 + c;
        if (ch0 >= p.k) break;  // warp-uniform
        if (kEpilogue != kPlain) {
          const int co = ch0 + lane;
          float m = 0.0f, a = 0.0f, b = 0.0f;
          if (co < p.k) {
            m = mean[co];
            a = rsqrtf(variance[co] + epsilon) * scale[co];
            b = bias[co];
          }
          prm[lane * 3 + 0] = m;
          prm[lane * 3 + 1] = a;
          prm[lane * 3 + 2] = b;
        }
        uint32_t accv[32];
        tmem_load_32x32(taddr + c, accv);
        __syncwarp();
        const int rows = min(32, p.k - ch0);
        float res[32];
        if (kEpilogue == kBatchNormAddRelu) {
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            res[j] = (valid && j < rows) ? __ldg(residual + base + static_cast<long long>(ch0 + j) * pixels_per_image)
                                         : 0.0f;
          }
        }
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          if (valid && j < rows) {
            float v = __uint_as_float(accv[j]);
            if (kEpilogue != kPlain) v = (v - prm[j * 3 + 0]) * prm[j * 3 + 1] + prm[j * 3 + 2];
            if (kEpilogue == kBatchNormAddRelu) v += res[j];
            if (kEpilogue == kBatchNormRelu || kEpilogue == kBatchNormAddRelu) v = fmaxf(v, 0.0f);
            out[base + static_cast<long long>(ch0 + j) * pixels_per_image] = v;
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

template <int kEpilogue>
__device__ __forceinline__ void conv_tm_dispatch(const TmaDescriptor* tma_w, const float* x, const float* scale,
                                                 const float* bias, const float* mean, const float* variance,
                                                 const float* residual, float* out, const ConvShape& p,
                                                 float epsilon, void* scratch) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
  if (p.k <= 64) {
    conv_tm<kEpilogue, 64>(smem, tma_w, x, scale, bias, mean, variance, residual, out, p, epsilon, scratch);
  } else {
    conv_tm<kEpilogue, 128>(smem, tma_w, x, scale, bias, mean, variance, residual, out, p, epsilon, scratch);
  }
}

}  // namespace

#define CTB_CONV_DIMS                                                                                 \
  int n, int c, int h, int w, int k, int r, int s, int out_h, int out_w, int stride_h, int stride_w, \
      int pad_h, int pad_w, int dilation_h, int dilation_w
#define CTB_CONV_SHAPE \
  ConvShape{n, c, h, w, k, r, s, out_h, out_w, stride_h, stride_w, pad_h, pad_w, dilation_h, dilation_w}

extern "C" __global__ void __launch_bounds__(kThreads, 1)
ctb_conv_f32_tm(const __grid_constant__ TmaDescriptor tma_w, const float* x, float* output, CTB_CONV_DIMS,
                CTB_RESERVED_PARAMS) {
  (void)profile_scratch;
  conv_tm_dispatch<kPlain>(&tma_w, x, nullptr, nullptr, nullptr, nullptr, nullptr, output, CTB_CONV_SHAPE, 0.0f,
                           runtime_scratch);
}

extern "C" __global__ void __launch_bounds__(kThreads, 1)
ctb_conv_bn_f32_tm(const __grid_constant__ TmaDescriptor tma_w, const float* x, const float* scale,
                   const float* bias, const float* mean, const float* variance, float* output, CTB_CONV_DIMS,
                   float epsilon, CTB_RESERVED_PARAMS) {
  (void)profile_scratch;
  conv_tm_dispatch<kBatchNorm>(&tma_w, x, scale, bias, mean, variance, nullptr, output, CTB_CONV_SHAPE, epsilon,
                               runtime_scratch);
}

extern "C" __global__ void __launch_bounds__(kThreads, 1)
ctb_conv_bn_relu_f32_tm(const __grid_constant__ TmaDescriptor tma_w, const float* x, const float* scale,
                        const float* bias, const float* mean, const float* variance, float* output,
                        CTB_CONV_DIMS, float epsilon, CTB_RESERVED_PARAMS) {
  (void)profile_scratch;
  conv_tm_dispatch<kBatchNormRelu>(&tma_w, x, scale, bias, mean, variance, nullptr, output, CTB_CONV_SHAPE,
                                   epsilon, runtime_scratch);
}

extern "C" __global__ void __launch_bounds__(kThreads, 1)
ctb_conv_bn_add_relu_f32_tm(const __grid_constant__ TmaDescriptor tma_w, const float* x, const float* scale,
                            const float* bias, const float* mean, const float* variance, const float* residual,
                            float* output, CTB_CONV_DIMS, float epsilon, CTB_RESERVED_PARAMS) {
  (void)profile_scratch;
  conv_tm_dispatch<kBatchNormAddRelu>(&tma_w, x, scale, bias, mean, variance, residual, output, CTB_CONV_SHAPE,
                                      epsilon, runtime_scratch);
}
