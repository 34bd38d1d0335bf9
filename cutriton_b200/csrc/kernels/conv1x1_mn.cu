// FP32 1x1 / stride-1 / unpadded convolution (+BatchNorm [+residual]
// [+ReLU]) as a 3xTF32 tcgen05 GEMM with the output channels on M:
//
//   D[co, px] = sum_ci W[co, ci] . X[n, ci, px]      (px = h * W + w of image n)
//
// the math of the reference's conv kernels (python/cutriton/triton_kernels/
// resnet.py:41-47 BatchNorm folding, :216-400 fused conv entry points) for
// the NCHW 1x1 layers. In NCHW the activation plane of one input channel is
// contiguous along px, so X is an MN-major B operand that TMA copies straight
// from global memory ({32 px, 32 ci} boxes, 128-byte swizzle with 32-byte
// atoms) — no gather — and the output of one channel is contiguous along px
// too: the epilogue thread of TMEM lane co holds 32 consecutive pixels of
// its channel and leaves them through a {32 px, 32 co} tensor store.
//
// 3xTF32: W arrives prepacked as exact TF32 hi / lo planes
// (conv_w_tf32x2_cb); four split warps turn each landed X block into
// X_hi = X with the low 13 mantissa bits cleared (in place) and
// X_lo = X - X_hi (a second buffer of the same layout), and the issuer runs
// D += W_hi.X_hi + W_lo.X_hi + W_hi.X_lo per 8-channel step.
//
// Tiles: 128 output channels x 128 pixels of one image (the last pixel tile
// of an image is partly outside it: TMA zero-fills those loads and clips
// those stores), channel tile fastest so neighbouring CTAs share X through
// L2. Persistent: CTA b takes tiles b, b + grid, ...
//
// Warps (320 threads): 0 — TMA producer (W_hi, W_lo, four X boxes per
// 32-channel k block); 1 — TMEM owner and MMA issuer; 2-5 — split warps;
// 6-9 — epilogue, one per TMEM lane quarter (warp % 4), each with its own
// residual ring (loaded three chunks ahead) and two output boxes. Two TMEM
// accumulators (2 x 128 columns) let the epilogue of tile i overlap the MMAs
// of tile i + 1. Every wait is bounded (tc_common.cuh).

#include "tc_common.cuh"

namespace {

using namespace ctb::tc;

constexpr int kBM = 128;  // output channels per tile (TMEM lanes)
constexpr int kBN = 128;  // pixels per tile (TMEM columns)
constexpr int kBK = 32;   // input channels per k block
constexpr int kMaxStages = 3;
constexpr int kSplitWarp0 = 2;
constexpr int kSplitThreads = 128;
constexpr int kEpiWarp0 = 6;
constexpr int kEpiWarps = 4;
constexpr int kThreads = (kEpiWarp0 + kEpiWarps) * 32;
constexpr uint32_t kWPlane = kBM * kBK * 4;  // 16 KB: W_hi or W_lo, K-major rows of 128 B
constexpr uint32_t kBox = 32 * 32 * 4;        // 4 KB: {32 px, 32 channels}, rows of 128 B
constexpr uint32_t kXBytes = (kBN / 32) * kBox;  // 16 KB: four pixel boxes of one k block
constexpr uint32_t kStageBytes = 2 * kWPlane + 2 * kXBytes;
constexpr int kMaxResSlots = 4;
constexpr int kResAhead = 3;
constexpr int kOutSlots = 2;
constexpr uint32_t kTmemCols = 2 * kBN;
constexpr int kChunks = kBN / 32;  // 32-pixel chunks per tile

enum Epilogue { kPlain = 0, kBatchNorm = 1, kBatchNormRelu = 2, kBatchNormAddRelu = 3 };

// Stages and epilogue boxes per kernel: with a residual, each epilogue warp
// keeps a 4-slot residual ring (loads three chunks ahead) besides its two
// output boxes, which leaves room for two 64 KB stages; without one, three
// stages fit.
template <int kEpilogue>
struct Config {
  static constexpr bool kResidual = kEpilogue == kBatchNormAddRelu;
  static constexpr int kStages = kResidual ? 2 : 3;
  static constexpr int kResSlots = kResidual ? kMaxResSlots : 0;
  static constexpr uint32_t kEpiBytes = (kResSlots + kOutSlots) * kBox;  // per epilogue warp
};

struct __align__(8) Barriers {
  uint64_t full[kMaxStages];   // W and X of the stage landed
  uint64_t ready[kMaxStages];  // X_hi / X_lo written by the split warps
  uint64_t empty[kMaxStages];  // the stage's MMAs completed
  uint64_t tmem_full[2];
  uint64_t tmem_empty[2];
  uint64_t res_full[kEpiWarps][kMaxResSlots];
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
};

template <int kEpilogue>
constexpr uint32_t smem_bytes() {
  using C = Config<kEpilogue>;
  return C::kStages * kStageBytes + kEpiWarps * C::kEpiBytes + sizeof(Barriers) + 1024;
}
static_assert(smem_bytes<kBatchNormRelu>() <= 232448 && smem_bytes<kBatchNormAddRelu>() <= 232448,
              "shared memory budget");

// MN-major TF32 operand in the "128-byte swizzle, 32-byte atom" canonical
// layout (the one layout the tensor core takes for MN-major TF32; layout
// type 1): rows of 128 B (32 TF32 along MN) whose 32-byte chunks are permuted
// by row % 4 — what a TMA copy with CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B
// writes — 4-row groups along K 512 B apart (SBO), 32-element MN atoms `lbo`
// bytes apart (LBO).
__device__ __forceinline__ uint64_t smem_desc_mnmajor_sw128_32b(const void* tile, uint32_t lbo) {
  const uint64_t start = (smem_addr(tile) >> 4) & 0x3FFFu;
  const uint64_t sbo = 512 >> 4;
  return start | (static_cast<uint64_t>(lbo >> 4) << 16) | (sbo << 32) | (1ull << 46) | (1ull << 61);
}

// kind::tf32, FP32 accumulator, A K-major, B MN-major, M = 128, N = 128.
constexpr uint32_t kInstrDesc = instr_desc(kFormatTF32, kBM, kBN) | (1u << 16);

__device__ __forceinline__ void tma_store_3d(const TmaDescriptor* desc, const void* src, int x, int y, int z) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(desc)),
               "r"(smem_addr(src)), "r"(x), "r"(y), "r"(z)
               : "memory");
}

struct Shape {
  int n, c, hw, k;
};

template <int kEpilogue>
__device__ __forceinline__ void conv1x1_mn(const TmaDescriptor* tma_w, const TmaDescriptor* tma_x,
                                           const TmaDescriptor* tma_out, const TmaDescriptor* tma_res,
                                           const float* __restrict__ x, const float* __restrict__ scale,
                                           const float* __restrict__ bias, const float* __restrict__ mean,
                                           const float* __restrict__ variance, const float* __restrict__ residual,
                                           float* __restrict__ out, const Shape& p, float epsilon, void* scratch) {
  constexpr int kStages = Config<kEpilogue>::kStages;
  constexpr int kResSlots = Config<kEpilogue>::kResSlots;
  constexpr int kResMod = kResSlots > 0 ? kResSlots : 1;  // slot arithmetic (residual kernels only)
  constexpr uint32_t kEpiBytes = Config<kEpilogue>::kEpiBytes;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
  uint8_t* epi = smem + kStages * kStageBytes;
  Barriers* bars = reinterpret_cast<Barriers*>(epi + kEpiWarps * kEpiBytes);
  volatile int* abort = &bars->abort;
  auto w_hi = [&](int s) { return smem + s * kStageBytes; };
  auto w_lo = [&](int s) { return smem + s * kStageBytes + kWPlane; };
  auto x_hi = [&](int s) { return smem + s * kStageBytes + 2 * kWPlane; };
  auto x_lo = [&](int s) { return smem + s * kStageBytes + 2 * kWPlane + kXBytes; };

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  // Contract (checked by the pack's constraints, re-checked here): C a
  // multiple of 32, H*W a multiple of 4 and 16-byte aligned tensors (the
  // tensor maps exist exactly then).
  const bool aligned = (reinterpret_cast<uintptr_t>(x) & 15) == 0 && (reinterpret_cast<uintptr_t>(out) & 15) == 0 &&
                       (kEpilogue != kBatchNormAddRelu || (reinterpret_cast<uintptr_t>(residual) & 15) == 0);
  if (p.c % kBK != 0 || p.hw % 4 != 0 || !aligned) {
    if (threadIdx.x == 0) ctb::report_error(scratch, ctb::kErrorBadShape, 70);
    return;
  }
  const int k_blocks = p.c / kBK;
  const int px_tiles = (p.hw + kBN - 1) / kBN;
  const int co_tiles = (p.k + kBM - 1) / kBM;
  const long long tiles = static_cast<long long>(p.n) * px_tiles * co_tiles;
  const int my_tiles = tiles > blockIdx.x ? static_cast<int>((tiles - 1 - blockIdx.x) / gridDim.x) + 1 : 0;
  struct TilePos {
    int co0, px0, img;
  };
  auto tile_pos = [&](int local) {
    const long long t = blockIdx.x + static_cast<long long>(local) * gridDim.x;
    const long long rest = t / co_tiles;
    return TilePos{static_cast<int>(t - rest * co_tiles) * kBM, static_cast<int>(rest % px_tiles) * kBN,
                   static_cast<int>(rest / px_tiles)};
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bars->full[s], 1);
      mbar_init(&bars->ready[s], kSplitThreads);
      mbar_init(&bars->empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&bars->tmem_full[b], 1);
      mbar_init(&bars->tmem_empty[b], kEpiWarps);
    }
    for (int w = 0; w < kEpiWarps; ++w) {
      for (int b = 0; b < kResSlots; ++b) mbar_init(&bars->res_full[w][b], 1);
    }
    mbar_init(&bars->drain, 1);
    bars->abort = 0;
    mbar_init_fence();
    tma_prefetch(tma_w);
    tma_prefetch(tma_x);
    tma_prefetch(tma_out);
    if (kEpilogue == kBatchNormAddRelu) tma_prefetch(tma_res);
  }
  if (warp == 1) tmem_alloc(&bars->tmem_base, kTmemCols);
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  const uint32_t tmem = bars->tmem_base;
  CTB_GRID_DEPENDENCY_SYNC();
  const int total_blocks = my_tiles * k_blocks;

  if (warp == 0 && lane == 0) {
    // ---- TMA producer ----
    int g = 0;
    bool stop = false;
    for (int local = 0; local < my_tiles && !stop; ++local) {
      const TilePos t = tile_pos(local);
      for (int kb = 0; kb < k_blocks; ++kb, ++g) {
        const int s = g % kStages;
        const int use = g / kStages;
        if (use > 0 && !mbar_wait(&bars->empty[s], (use - 1) & 1, abort, scratch, 71)) {
          stop = true;
          break;
        }
        mbar_arrive_expect_tx(&bars->full[s], 2 * kWPlane + kXBytes);
        tma_load_3d(w_hi(s), tma_w, &bars->full[s], kb * kBK, t.co0, 0);
        tma_load_3d(w_lo(s), tma_w, &bars->full[s], kb * kBK, t.co0, 1);
#pragma unroll
        for (int i = 0; i < kBN / 32; ++i) {
          tma_load_3d(x_hi(s) + i * kBox, tma_x, &bars->full[s], t.px0 + 32 * i, kb * kBK, t.img);
        }
      }
    }
    if (*abort) {
      // The newest copy of each stage may still be in flight: let it land
      // before shared memory is released (older ones were waited for).
      for (int q = g > kStages ? g - kStages : 0; q < g; ++q) {
        volatile int never = 0;
        mbar_wait(&bars->full[q % kStages], (q / kStages) & 1, &never, scratch, 72);
      }
    }
  } else if (warp == 1 && lane == 0) {
    // ---- MMA issuer ----
    int g = 0;
    bool ok = true;
    for (int local = 0; local < my_tiles && ok; ++local) {
      const int buf = local & 1;
      if (local >= 2 && !mbar_wait(&bars->tmem_empty[buf], ((local >> 1) - 1) & 1, abort, scratch, 73)) {
        ok = false;
        break;
      }
      tc_fence_after_sync();
      const uint32_t acc = tmem + buf * kBN;
      for (int kb = 0; kb < k_blocks; ++kb, ++g) {
        const int s = g % kStages;
        // full: the weight copies landed (the split warps saw it too); ready:
        // X_hi / X_lo are written.
        if (!mbar_wait(&bars->full[s], (g / kStages) & 1, abort, scratch, 80) ||
            !mbar_wait(&bars->ready[s], (g / kStages) & 1, abort, scratch, 74)) {
          ok = false;
          break;
        }
        tc_fence_after_sync();
        const uint64_t a_hi = smem_desc_kmajor_sw128(w_hi(s));
        const uint64_t a_lo = smem_desc_kmajor_sw128(w_lo(s));
        const uint64_t b_hi = smem_desc_mnmajor_sw128_32b(x_hi(s), kBox);
        const uint64_t b_lo = smem_desc_mnmajor_sw128_32b(x_lo(s), kBox);
#pragma unroll
        for (int kk = 0; kk < kBK / 8; ++kk) {
          // 8 input channels per UMMA: +32 bytes along A's rows, +1024 bytes
          // (two 4-row groups) down B.
          const uint64_t da = 2 * kk, db = 64 * kk;
          umma_tf32(acc, a_hi + da, b_hi + db, kInstrDesc, (kb | kk) != 0);
          umma_tf32(acc, a_lo + da, b_hi + db, kInstrDesc, 1);
          umma_tf32(acc, a_hi + da, b_lo + db, kInstrDesc, 1);
        }
        umma_commit(&bars->empty[s]);
      }
      if (ok) umma_commit(&bars->tmem_full[buf]);
    }
    if (!ok) {
      umma_commit(&bars->drain);
      volatile int never = 0;
      mbar_wait(&bars->drain, 0, &never, scratch, 75);
    }
  } else if (warp >= kSplitWarp0 && warp < kSplitWarp0 + kSplitThreads / 32) {
    // ---- split warps: X -> X_hi (in place) and X_lo ----
    const int tid = threadIdx.x - kSplitWarp0 * 32;
    for (int g = 0; g < total_blocks; ++g) {
      const int s = g % kStages;
      if (!mbar_wait(&bars->full[s], (g / kStages) & 1, abort, scratch, 76)) break;
      float4* hi = reinterpret_cast<float4*>(x_hi(s));
      float4* lo = reinterpret_cast<float4*>(x_lo(s));
#pragma unroll
      for (int j = 0; j < static_cast<int>(kXBytes / 16) / kSplitThreads; ++j) {
        const int i = tid + j * kSplitThreads;
        const float4 v = hi[i];
        float4 h, l;
        h.x = __uint_as_float(__float_as_uint(v.x) & 0xFFFFE000u);
        h.y = __uint_as_float(__float_as_uint(v.y) & 0xFFFFE000u);
        h.z = __uint_as_float(__float_as_uint(v.z) & 0xFFFFE000u);
        h.w = __uint_as_float(__float_as_uint(v.w) & 0xFFFFE000u);
        l.x = v.x - h.x;
        l.y = v.y - h.y;
        l.z = v.z - h.z;
        l.w = v.w - h.w;
        hi[i] = h;
        lo[i] = l;
      }
      // Generic-proxy writes become visible to the tensor core's reads.
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      mbar_arrive(&bars->ready[s]);
    }
  } else if (warp >= kEpiWarp0) {
    // ---- epilogue: TMEM lane quarter q = warp % 4, thread = output channel ----
    const int q = warp & 3;
    const int ew = warp - kEpiWarp0;
    uint8_t* res_ring = epi + ew * kEpiBytes;
    uint8_t* out_ring = res_ring + kResSlots * kBox;
    const int total_chunks = my_tiles * kChunks;
    // Residual of chunk h (32 pixels of this warp's 32 channels) into slot
    // h % kResSlots; lane 0 issues, the slot's barrier counts the bytes.
    auto load_residual = [&](int h) {
      if (kEpilogue != kBatchNormAddRelu || h >= total_chunks || lane != 0) return;
      const TilePos t = tile_pos(h / kChunks);
      const int slot = h % kResMod;
      mbar_arrive_expect_tx(&bars->res_full[ew][slot], kBox);
      tma_load_3d(res_ring + slot * kBox, tma_res, &bars->res_full[ew][slot], t.px0 + 32 * (h % kChunks),
                  t.co0 + 32 * q, t.img);
    };
    for (int h = 0; h < kResAhead; ++h) load_residual(h);
    int res_landed = 0;  // residual chunks known to have landed (all before it too)
    float pm = 0.0f, pa = 0.0f, pb = 0.0f;
    int params_co0 = -1;
    bool failed = false;
    for (int local = 0; local < my_tiles && !failed; ++local) {
      const int buf = local & 1;
      const TilePos t = tile_pos(local);
      const int co = t.co0 + 32 * q + lane;
      if (kEpilogue != kPlain && t.co0 != params_co0) {
        params_co0 = t.co0;
        pm = pa = pb = 0.0f;
        if (co < p.k) {
          pm = mean[co];
          pa = rsqrtf(variance[co] + epsilon) * scale[co];
          pb = bias[co];
        }
      }
      const bool ready = mbar_wait(&bars->tmem_full[buf], (local >> 1) & 1, abort, scratch, 77);
      __syncwarp();
      if (!ready) break;
      tc_fence_after_sync();
      const uint32_t taddr = tmem + buf * kBN + (static_cast<uint32_t>(q * 32) << 16);
      for (int c = 0; c < kChunks; ++c) {
        const int h = local * kChunks + c;
        uint32_t v[32];
        tmem_load_32x32(taddr + 32 * c, v);
        if (c == kChunks - 1) {
          // This warp's accumulator rows are in registers: release them.
          tc_fence_before_sync();
          __syncwarp();
          if (lane == 0) mbar_arrive(&bars->tmem_empty[buf]);
        }
        const float4* res_row = reinterpret_cast<const float4*>(res_ring + (h % kResMod) * kBox + lane * 128);
        if (kEpilogue == kBatchNormAddRelu) {
          const bool landed = mbar_wait(&bars->res_full[ew][h % kResMod], (h / kResMod) & 1, abort, scratch, 78);
          __syncwarp();
          if (!landed) {
            failed = true;  // recorded; the copies in flight are drained below
            break;
          }
          res_landed = h + 1;
        }
        // Output box slot: the store issued from it two chunks ago must have
        // been read out.
        uint8_t* out_box = out_ring + (h % kOutSlots) * kBox;
        if (h >= kOutSlots && lane == 0) asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(kOutSlots - 1) : "memory");
        __syncwarp();
        float4* out_row = reinterpret_cast<float4*>(out_box + lane * 128);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          // 16-byte chunk j of row `lane` sits at chunk j ^ (lane % 8) (128-byte swizzle).
          const int phys = j ^ (lane & 7);
          float r[4] = {0.0f, 0.0f, 0.0f, 0.0f};
          if (kEpilogue == kBatchNormAddRelu) {
            const float4 rv = res_row[phys];
            r[0] = rv.x;
            r[1] = rv.y;
            r[2] = rv.z;
            r[3] = rv.w;
          }
          float o[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            float a = __uint_as_float(v[4 * j + e]);
            if (kEpilogue != kPlain) a = (a - pm) * pa + pb;
            if (kEpilogue == kBatchNormAddRelu) a += r[e];
            if (kEpilogue == kBatchNormRelu || kEpilogue == kBatchNormAddRelu) a = fmaxf(a, 0.0f);
            o[e] = a;
          }
          out_row[phys] = make_float4(o[0], o[1], o[2], o[3]);
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if (lane == 0) {
          tma_store_3d(tma_out, out_box, t.px0 + 32 * c, t.co0 + 32 * q, t.img);
          asm volatile("cp.async.bulk.commit_group;" ::: "memory");
        }
        // Slot (h + kResAhead) % kResSlots held chunk h - 1's residual, read
        // by every lane before the __syncwarp above.
        load_residual(h + kResAhead);
      }
    }
    if (lane == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
    if (kEpilogue == kBatchNormAddRelu && lane == 0) {
      // Residual copies issued for chunks this warp did not consume (abort)
      // must land before shared memory is released: chunks below res_landed
      // have; the kResAhead after it were issued.
      for (int h = res_landed; h < total_chunks && h < res_landed + kResAhead; ++h) {
        volatile int never = 0;
        mbar_wait(&bars->res_full[ew][h % kResMod], (h / kResMod) & 1, &never, scratch, 79);
      }
    }
  }
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  if (warp == 1) tmem_dealloc(tmem, kTmemCols);
}

}  // namespace

#define CTB_MN_DIMS int n, int c, int h, int w, int k
#define CTB_MN_SHAPE Shape{n, c, h * w, k}

extern "C" __global__ void __launch_bounds__(kThreads, 1)
ctb_conv1x1_f32_mn(const __grid_constant__ TmaDescriptor tma_w, const __grid_constant__ TmaDescriptor tma_x,
                   const __grid_constant__ TmaDescriptor tma_out, const float* x, float* output, CTB_MN_DIMS,
                   CTB_RESERVED_PARAMS) {
  (void)profile_scratch;
  conv1x1_mn<kPlain>(&tma_w, &tma_x, &tma_out, nullptr, x, nullptr, nullptr, nullptr, nullptr, nullptr, output,
                     CTB_MN_SHAPE, 0.0f, runtime_scratch);
}

extern "C" __global__ void __launch_bounds__(kThreads, 1)
ctb_conv1x1_bn_f32_mn(const __grid_constant__ TmaDescriptor tma_w, const __grid_constant__ TmaDescriptor tma_x,
                      const __grid_constant__ TmaDescriptor tma_out, const float* x, const float* scale,
                      const float* bias, const float* mean, const float* variance, float* output, CTB_MN_DIMS,
                      float epsilon, CTB_RESERVED_PARAMS) {
  (void)profile_scratch;
  conv1x1_mn<kBatchNorm>(&tma_w, &tma_x, &tma_out, nullptr, x, scale, bias, mean, variance, nullptr, output,
                         CTB_MN_SHAPE, epsilon, runtime_scratch);
}

extern "C" __global__ void __launch_bounds__(kThreads, 1)
ctb_conv1x1_bn_relu_f32_mn(const __grid_constant__ TmaDescriptor tma_w, const __grid_constant__ TmaDescriptor tma_x,
                           const __grid_constant__ TmaDescriptor tma_out, const float* x, const float* scale,
                           const float* bias, const float* mean, const float* variance, float* output, CTB_MN_DIMS,
                           float epsilon, CTB_RESERVED_PARAMS) {
  (void)profile_scratch;
  conv1x1_mn<kBatchNormRelu>(&tma_w, &tma_x, &tma_out, nullptr, x, scale, bias, mean, variance, nullptr, output,
                             CTB_MN_SHAPE, epsilon, runtime_scratch);
}

extern "C" __global__ void __launch_bounds__(kThreads, 1)
ctb_conv1x1_bn_add_relu_f32_mn(const __grid_constant__ TmaDescriptor tma_w,
                               const __grid_constant__ TmaDescriptor tma_x,
                               const __grid_constant__ TmaDescriptor tma_out,
                               const __grid_constant__ TmaDescriptor tma_res, const float* x, const float* scale,
                               const float* bias, const float* mean, const float* variance, const float* residual,
                               float* output, CTB_MN_DIMS, float epsilon, CTB_RESERVED_PARAMS) {
  (void)profile_scratch;
  conv1x1_mn<kBatchNormAddRelu>(&tma_w, &tma_x, &tma_out, &tma_res, x, scale, bias, mean, variance, residual, output,
                                CTB_MN_SHAPE, epsilon, runtime_scratch);
}
