// FP32 convolution (+BatchNorm [+residual] [+ReLU]) as a 3xTF32 implicit
// GEMM on the 5th-generation tensor cores with the activation operand held in
// tensor memory (TMEM), NCHW / OIHW.
//
// GEMM view: D[pixel, co] = sum_k X_im2col[pixel, k] * W[co, k]. When
// C % 32 == 0 the k blocks walk the filter taps inside each 32-channel block,
// k = ((c / 32) * R * S + r * S + s) * 32 + c % 32, so successive blocks of a
// pixel tile read the same 32 channel planes shifted by one tap (L1 hits);
// otherwise k = (r * S + s) * Cp + c with Cp = C rounded up to a multiple of 4
// (padded channels carry zero weights) and a per-CTA table in shared memory
// maps each 4-wide k chunk to its (r, s, c). FP32 accuracy from TF32
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
// Pixel tiles are either flat over N*H*W or (1x1 variant) aligned to images.
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
// Gather groups of four warps (one per TMEM lane quarter) taking k blocks in
// turn: two when the blocks come from global loads, one suffices when they
// arrive by TMA (and leaves 168 registers per thread instead of 128).
#ifndef CTB_TM_GATHER_GROUPS
#define CTB_TM_GATHER_GROUPS 2
#endif
constexpr int kGatherGroups = CTB_TM_GATHER_GROUPS;
// Epilogue warps: 4 (one per TMEM lane quarter), or 8 — two sets of four
// ("halves") taking alternate 32-channel chunks, each with its own named
// barrier, staging slots and copy-issuing threads.
#ifndef CTB_TM_EPI_WARPS
#define CTB_TM_EPI_WARPS 4
#endif
constexpr int kEpiWarps = CTB_TM_EPI_WARPS;
constexpr int kHalves = kEpiWarps / 4;
static_assert(kEpiWarps == 4 || kEpiWarps == 8, "epilogue warps");

constexpr int kThreads = (2 + kEpiWarps + 4 * kGatherGroups) * 32;
constexpr int kEpilogueWarp0 = 2;
constexpr int kGatherWarp0 = kEpilogueWarp0 + kEpiWarps;
constexpr int kGroupThreads = 128;    // four warps, one per lane quarter
constexpr int kBoxRows = 64;          // weight rows (output channels) per TMA box
constexpr uint32_t kBoxBytes = kBoxRows * kBK * 4;  // 8 KB
constexpr uint32_t kTmemCols = 512;
// Pipeline depths (compile-time; the pack's shared-memory size follows them).
#ifndef CTB_TM_STAGES_N128
#define CTB_TM_STAGES_N128 4
#endif
#ifndef CTB_TM_STAGES_N64
#define CTB_TM_STAGES_N64 6
#endif
#ifndef CTB_TM_SLOTS
#define CTB_TM_SLOTS 6
#endif
#ifndef CTB_TM_LOAD_AHEAD
#define CTB_TM_LOAD_AHEAD 4
#endif
// 1 (the 1x1 variant): 1x1 / stride-1 / unpadded convolutions load each k
// block of a tile that lies in one image with one TMA tensor copy ({128
// pixels, 32 channels} of the [N][C][H*W] view) into a shared-memory ring;
// the gather warps read it from there instead of issuing 32 global loads per
// pixel. Other tiles and shapes use the global-load gather.
#ifndef CTB_TM_A_TMA
#define CTB_TM_A_TMA 0
#endif
// 1: pixel tiles never straddle images (ceil(H*W / 128) tiles per image, the
// last one partly empty) whenever H*W is a multiple of 4, so every tile takes
// the single-tensor-copy paths. 0: flat tiling over N*H*W pixels.
#ifndef CTB_TM_IMAGE_TILES
#define CTB_TM_IMAGE_TILES 0
#endif
// 1 (the small-channel variant, e.g. the 7x7/2 ResNet stem): per pixel tile,
// the whole input window its im2col touches — box {kWinW columns from -4,
// kWinH rows from the tile's first input row, 4 channels, 1 image} of the
// NCHW input — arrives with one TMA copy into one of two shared-memory
// buffers, and the gather reads every tap from there with no bounds checks
// (TMA zero-fills outside the image). Tiles whose window does not fit, or
// that straddle two images, use the global-load gather.
#ifndef CTB_TM_WINDOW
#define CTB_TM_WINDOW 0
#endif
// 1: 64-channel tiles issue 2 instead of 3 UMMAs per 8 k: A_hi . [B_hi; B_lo]
// (N = 128 over the stacked hi / lo weight planes, which sit contiguously in
// shared memory) into a 128-column accumulator, then A_lo . B_hi (N = 64)
// accumulated into its first 64 columns (the tensor pipe runs them in
// order); the epilogue adds the two halves. Fewer, wider instructions for a
// pipe bound by per-instruction cost, in the same TMEM as the 3-UMMA form.
#ifndef CTB_TM_SPLIT_N
#define CTB_TM_SPLIT_N 0
#endif
// 1: the same for 128-channel tiles (A_hi . [B_hi; B_lo] as one N = 256
// UMMA); the 256-column accumulator then fits once, so the epilogue of a tile
// no longer overlaps the next tile's MMAs.
#ifndef CTB_TM_SPLIT_N128
#define CTB_TM_SPLIT_N128 0
#endif
constexpr int kMaxStages = 6;
constexpr uint32_t kStageRegionBytes =
    CTB_TM_STAGES_N128 * 32768 > CTB_TM_STAGES_N64 * 16384 ? CTB_TM_STAGES_N128 * 32768 : CTB_TM_STAGES_N64 * 16384;
constexpr int kChunkTable = 256;                     // 4-wide k chunks described in shared memory
// Epilogue staging ring: kSlots slots of [32 channels][128 pixels] FP32; the
// residual is loaded kLoadAhead chunks ahead, so a slot is refilled two
// chunks after its store was issued.
constexpr int kSlots = CTB_TM_SLOTS;
constexpr int kLoadAhead = CTB_TM_LOAD_AHEAD;
static_assert(kSlots <= 6 && kLoadAhead < kSlots && kSlots >= 4, "staging ring");
// Chunk h belongs to half h % kHalves; so must chunk h + kLoadAhead and every
// chunk that reuses slot h % kSlots.
static_assert(kLoadAhead % kHalves == 0 && kSlots % kHalves == 0, "staging ring per half");
constexpr uint32_t kStagingBytes = kSlots * 32 * 128 * 4;
// Activation blocks in flight (1x1 variant). A multiple of the gather group
// count, so each slot is only ever used by one gather group: a group
// then waits on a slot's phases strictly in order. With an odd ring the other
// group could reach a slot's next use while its current phase is still open,
// and a parity wait would mistake the previous completed phase for it.
#ifndef CTB_TM_A_RING
#define CTB_TM_A_RING 4
#endif
constexpr int kARing = CTB_TM_A_RING;
static_assert(kARing % kGatherGroups == 0, "activation ring slots must belong to one gather group");
// The register-path epilogue (H*W not a multiple of 4) assumes one half.
static_assert(kEpiWarps == 4 || CTB_TM_A_TMA, "8 epilogue warps need the 1x1 variant's fallback");
constexpr uint32_t kARingBytes = CTB_TM_A_TMA ? kARing * 32 * 128 * 4 : 0;
constexpr int kWinW = 232, kWinH = 11, kWinC = 4;
constexpr uint32_t kWinBytes = kWinW * kWinH * kWinC * 4;
static_assert(kWinBytes % 128 == 0, "window buffers keep 128-byte alignment");

template <int BN>
struct Tile {
  // Weight stages in shared memory (pack option) and activation stages in
  // TMEM (all the columns the two accumulators leave: 4 for BN = 128, 6 for
  // BN = 64) are separate rings with separate "empty" barriers.
  static constexpr int kStages = BN == 64 ? CTB_TM_STAGES_N64 : CTB_TM_STAGES_N128;
  static_assert(kStages <= kMaxStages, "stage count");
  static constexpr uint32_t kPlaneBytes = BN * kBK * 4;  // one of hi / lo
  static constexpr uint32_t kStageBytes = 2 * kPlaneBytes;
  static constexpr bool kSplitN = (CTB_TM_SPLIT_N && BN == 64) || (CTB_TM_SPLIT_N128 && BN == 128);
  static constexpr uint32_t kAccCols = kSplitN ? 2 * BN : BN;  // one accumulator buffer
  static constexpr int kAccBufs = kAccCols * 2 <= 256 ? 2 : 1;   // double-buffered when it fits
  static constexpr uint32_t kAColumn0 = kAccBufs * kAccCols;    // first activation stage column
  static constexpr int kAStages = (kTmemCols - kAColumn0) / (2 * kBK);
  static_assert(kAStages <= kMaxStages && kAStages % 2 == 0, "activation stages (one gather group each)");
  static_assert(kStages * kStageBytes <= kStageRegionBytes, "shared memory budget");
};

enum Epilogue { kPlain = 0, kBatchNorm = 1, kBatchNormRelu = 2, kBatchNormAddRelu = 3 };

struct ConvShape {
  int n, c, h, w, k, r, s, out_h, out_w, stride_h, stride_w, pad_h, pad_w, dil_h, dil_w;
};

struct __align__(8) Barriers {
  uint64_t full_a[kMaxStages];
  uint64_t full_b[kMaxStages];
  uint64_t empty_a[kMaxStages];  // TMEM activation stage consumed by the MMAs
  uint64_t empty_b[kMaxStages];  // shared-memory weight stage consumed by the MMAs
  uint64_t tmem_full[2];
  uint64_t tmem_empty[2];
  uint64_t residual_full[6];  // bulk residual loads, one per staging slot
  uint64_t a_full[kARing];    // activation ring (1x1 variant): TMA landed / no-copy arrival
  uint64_t a_empty[kARing];   // activation ring: the gather group has read the block
  uint64_t win_full[2];       // input windows (small-channel variant)
  uint64_t win_empty[2];
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
  int consumed;
};
constexpr uint32_t kBarrierBytes = 512;
static_assert(sizeof(Barriers) <= kBarrierBytes, "barrier block");

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

// Named barrier 1 + half over the four warps of one epilogue half.
__device__ __forceinline__ void epilogue_bar(int half) {
  asm volatile("bar.sync %0, 128;" ::"r"(1 + half) : "memory");
}

// OR of `pred` over the four warps of an epilogue half; all get the same answer.
__device__ __forceinline__ bool epilogue_any(int half, bool pred) {
  int r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.b32 p, %1, 0;\n\t"
      "bar.red.or.pred q, %2, 128, p;\n\t"
      "selp.b32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(static_cast<int>(pred)), "r"(1 + half)
      : "memory");
  return r != 0;
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

// Predicated read-only load, kept in program order (asm volatile) so each
// block's loads are issued a whole block ahead of their use.
__device__ __forceinline__ float load_or_zero(const float* ptr, bool pred) {
  float v;
  asm volatile(
      "{\n\t.reg .pred q;\n\t"
      "setp.ne.b32 q, %2, 0;\n\t"
      "mov.b32 %0, 0;\n\t"
      "@q ld.global.nc.f32 %0, [%1];\n\t}"
      : "=f"(v)
      : "l"(ptr), "r"(static_cast<int>(pred)));
  return v;
}

// (r, s, c) of a 4-wide k chunk, packed c << 20 | r << 10 | s; -1 past kdim.
__device__ __forceinline__ int chunk_entry(int k, int cp, int kdim, int s_dim) {
  if (k >= kdim) return -1;
  const int tap = k / cp;
  const int r = tap / s_dim;
  return ((k - tap * cp) << 20) | (r << 10) | (tap - r * s_dim);
}

// Loads the 32 k values of block `kb` for one pixel (im2col, zero padding).
__device__ __forceinline__ void gather_block(const PixelSource& px, const ConvShape& p, int cp, int kdim,
                                             long long plane, int kb, const int* table, float (&v)[kBK]) {
  if (p.c % kBK == 0) {
    // One filter tap, 32 consecutive channels of one channel block.
    const int taps = p.r * p.s;
    const int cb = kb / taps;
    const int tap = kb - cb * taps;
    const int r = tap / p.s;
    const int ih = px.ih0 + r * p.dil_h;
    const int iw = px.iw0 + (tap - r * p.s) * p.dil_w;
    const bool inside = px.valid && ih >= 0 && ih < p.h && iw >= 0 && iw < p.w;
    const float* src =
        px.image + static_cast<long long>(cb * kBK) * plane + static_cast<long long>(ih) * p.w + iw;
#pragma unroll
    for (int kk = 0; kk < kBK; ++kk) v[kk] = load_or_zero(src + kk * plane, inside);
  } else {
    // Chunks of 4 k: four channels of one tap (cp is a multiple of 4).
#pragma unroll
    for (int j = 0; j < kBK / 4; ++j) {
      int c, r, s_tap;
      bool in_k;
      if (table != nullptr) {
        const int e = table[kb * (kBK / 4) + j];
        in_k = e >= 0;
        c = e >> 20;
        r = (e >> 10) & 1023;
        s_tap = e & 1023;
      } else {
        const int k = kb * kBK + 4 * j;
        const int tap = k / cp;
        in_k = k < kdim;
        c = k - tap * cp;
        r = tap / p.s;
        s_tap = tap - r * p.s;
      }
      const int ih = px.ih0 + r * p.dil_h;
      const int iw = px.iw0 + s_tap * p.dil_w;
      const bool inside = px.valid && in_k && ih >= 0 && ih < p.h && iw >= 0 && iw < p.w;
      const float* src = px.image + static_cast<long long>(c) * plane + static_cast<long long>(ih) * p.w + iw;
#pragma unroll
      for (int i = 0; i < 4; ++i) v[4 * j + i] = load_or_zero(src + i * plane, inside && c + i < p.c);
    }
  }
}

template <int kEpilogue, int BN>
__device__ __forceinline__ void conv_tm(uint8_t* smem, const TmaDescriptor* tma_w, const TmaDescriptor* tma_out,
                                        const TmaDescriptor* tma_res, const TmaDescriptor* tma_x,
                                        const TmaDescriptor* tma_xwin, const float* __restrict__ x,
                                        const float* __restrict__ scale, const float* __restrict__ bias,
                                        const float* __restrict__ mean, const float* __restrict__ variance,
                                        const float* __restrict__ residual, float* __restrict__ out,
                                        const ConvShape& p, float epsilon, void* scratch) {
  using T = Tile<BN>;
  constexpr int kStages = T::kStages;
  constexpr int kAStages = T::kAStages;
  Barriers* bars = reinterpret_cast<Barriers*>(smem + kStageRegionBytes);
  int* chunk_table = reinterpret_cast<int*>(smem + kStageRegionBytes + kBarrierBytes);
  float* staging = reinterpret_cast<float*>(smem + kStageRegionBytes + kBarrierBytes + kChunkTable * 4);
  float* a_ring = staging + kStagingBytes / 4;
  float* windows = a_ring + kARingBytes / 4;
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
  // Pixel tile mt covers flat pixels [tile_p0(mt), tile_p0(mt) + tile_rows(mt)).
  const bool image_tiles = CTB_TM_IMAGE_TILES && pixels_per_image % 4 == 0;
  const long long tiles_per_image = (pixels_per_image + kBM - 1) / kBM;
  const long long m_tiles = image_tiles ? p.n * tiles_per_image : (total_pixels + kBM - 1) / kBM;
  auto tile_p0 = [&](long long mt) -> long long {
    if (!image_tiles) return mt * kBM;
    const long long img = mt / tiles_per_image;
    return img * pixels_per_image + (mt - img * tiles_per_image) * kBM;
  };
  auto tile_rows = [&](long long mt) -> int {
    if (!image_tiles) return static_cast<int>(min(static_cast<long long>(kBM), total_pixels - mt * kBM));
    return static_cast<int>(min(static_cast<long long>(kBM), pixels_per_image - (mt % tiles_per_image) * kBM));
  };
  const long long tiles = m_tiles * co_tiles;
  const int my_tiles = tiles > blockIdx.x ? static_cast<int>((tiles - 1 - blockIdx.x) / gridDim.x) + 1 : 0;
  // 1x1 variant: tiles of a 1x1 / stride-1 / unpadded convolution that lie in
  // one image take their activation blocks by TMA (tma_x is encoded exactly
  // when the planes are 16-byte aligned, which a_tma_shape checks too).
  const bool a_tma_shape = CTB_TM_A_TMA && p.r == 1 && p.s == 1 && p.stride_h == 1 && p.stride_w == 1 &&
                           p.pad_h == 0 && p.pad_w == 0 && p.c % kBK == 0 && (p.h * p.w) % 4 == 0 &&
                           (reinterpret_cast<uintptr_t>(x) & 15) == 0;
  auto tile_a_tma = [&](long long tile, int* hw0, int* img) {
    if (!a_tma_shape) return false;
    const long long p0 = tile_p0(tile / co_tiles);
    const long long im = p0 / pixels_per_image;
    *hw0 = static_cast<int>(p0 - im * pixels_per_image);
    *img = static_cast<int>(im);
    return *hw0 + tile_rows(tile / co_tiles) <= pixels_per_image;
  };
  // Bulk / tensor-copy epilogue: needs 16-byte aligned rows of every channel
  // plane, the same condition under which the host encodes tma_out / tma_res
  // (otherwise they are bound as zeros and must not be touched).
  const bool bulk_epilogue = pixels_per_image % 4 == 0 && (reinterpret_cast<uintptr_t>(out) & 15) == 0 &&
                             (kEpilogue != kBatchNormAddRelu || (reinterpret_cast<uintptr_t>(residual) & 15) == 0);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bars->full_b[s], 1);
      mbar_init(&bars->empty_b[s], 1);
    }
    for (int s = 0; s < kAStages; ++s) {
      mbar_init(&bars->full_a[s], kGroupThreads);
      mbar_init(&bars->empty_a[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&bars->tmem_full[b], 1);
      mbar_init(&bars->tmem_empty[b], kEpiWarps);
    }
    for (int b = 0; b < kSlots; ++b) mbar_init(&bars->residual_full[b], 32);  // 8 issuing lanes x 4 warps of a half
    for (int b = 0; b < kARing; ++b) {
      mbar_init(&bars->a_full[b], 1);
      mbar_init(&bars->a_empty[b], kGroupThreads);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&bars->win_full[b], 1);
      mbar_init(&bars->win_empty[b], kGatherGroups * kGroupThreads);
    }
    mbar_init(&bars->drain, 1);
    bars->abort = 0;
    bars->consumed = 0;
    mbar_init_fence();
    tma_prefetch(tma_w);
    if (a_tma_shape) tma_prefetch(tma_x);
    if (bulk_epilogue) {
      tma_prefetch(tma_out);
      if (kEpilogue == kBatchNormAddRelu) tma_prefetch(tma_res);
    }
  }
  // Small / ragged channel counts: describe every 4-wide k chunk once.
  const bool use_table = p.c % kBK != 0 && k_blocks * (kBK / 4) <= kChunkTable && cp < 4096 && p.r < 1024 &&
                         p.s < 1024;
  if (use_table) {
    for (int i = threadIdx.x; i < k_blocks * (kBK / 4); i += blockDim.x) chunk_table[i] = chunk_entry(4 * i, cp, kdim, p.s);
  }
  // Small-channel variant: the columns every tile touches, [-pad, (OW-1)*stride
  // - pad + (S-1)*dil], must lie in the window's [-4, kWinW - 4); rows are
  // checked per tile. The tensor map needs 16-byte aligned rows and base.
  const bool window_shape = CTB_TM_WINDOW && use_table && cp == kWinC && k_blocks >= kGatherGroups &&
                            p.pad_w <= 4 && (p.out_w - 1) * p.stride_w - p.pad_w + (p.s - 1) * p.dil_w < kWinW - 4 &&
                            p.w % 4 == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0;
  struct Window {
    bool ok;
    int img, ih_lo;
  };
  auto window_of = [&](long long tile) {
    Window win{false, 0, 0};
    if (!window_shape) return win;
    const long long mt = tile / co_tiles;
    const long long p0 = tile_p0(mt);
    const int rows = tile_rows(mt);
    const long long img = p0 / pixels_per_image;
    const int hw0 = static_cast<int>(p0 - img * pixels_per_image);
    if (hw0 + rows > pixels_per_image) return win;  // straddles two images
    const int oh_a = hw0 / p.out_w, oh_b = (hw0 + rows - 1) / p.out_w;
    const int ih_lo = oh_a * p.stride_h - p.pad_h;
    const int ih_hi = oh_b * p.stride_h - p.pad_h + (p.r - 1) * p.dil_h;
    if (ih_hi - ih_lo + 1 > kWinH) return win;
    win.ok = true;
    win.img = static_cast<int>(img);
    win.ih_lo = ih_lo;
    return win;
  };
  if (warp == 0) tmem_alloc(&bars->tmem_base, kTmemCols);
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  const uint32_t tmem = bars->tmem_base;
  // Activations are touched only after the preceding kernel has finished.
  CTB_GRID_DEPENDENCY_SYNC();

  if (warp >= kGatherWarp0) {
    // ---- gather: one thread per output pixel, alternate k blocks per group ----
    const int group = (warp - kGatherWarp0) / 4;
    const int row = (warp & 3) * 32 + lane;  // TMEM lane = pixel within the tile
    const uint32_t lane_bits = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const long long plane = static_cast<long long>(p.h) * p.w;
    const int items = my_tiles * k_blocks;  // this CTA's k blocks, in issue order
    int px_local = -1;
    PixelSource px_cached{x, 0, 0, false};
    int win_local = -1, win_base = -1;
    bool win_valid = false;
    // Returns false when the kernel is aborting (window wait abandoned).
    auto fetch = [&](int item, float (&v)[kBK]) -> bool {
      const int local = item / k_blocks;
      const int kb = item - local * k_blocks;
      const long long tile = blockIdx.x + static_cast<long long>(local) * gridDim.x;
      int hw0, img;
      if (tile_a_tma(tile, &hw0, &img)) return true;  // arrives by TMA; read in publish
      if (window_shape) {
        // Every tile passes its buffer through the window barriers (a
        // no-copy arrival when it uses the global-load gather), so each
        // group waits for the tile's window before its first item of the
        // tile and releases it after its last.
        const int wb = local & 1;
        const int first = local * k_blocks + ((group - local * k_blocks) % kGatherGroups + kGatherGroups) % kGatherGroups;
        const int last_end = (local + 1) * k_blocks;
        if (item == first &&
            !mbar_wait(&bars->win_full[wb], (local >> 1) & 1, abort, scratch, 43)) {
          return false;
        }
        // The tile's window and this pixel's offset in it change once per
        // tile; base < 0 marks a tile without a window (or a pixel past it).
        if (local != win_local) {
          win_local = local;
          const Window win = window_of(tile);
          win_base = -1;
          if (win.ok) {
            const long long mt = tile / co_tiles;
            const long long pixel = tile_p0(mt) + row;
            const int rem = static_cast<int>(pixel - static_cast<long long>(win.img) * pixels_per_image);
            const int oh = rem / p.out_w;
            const int ow = rem - oh * p.out_w;
            win_base = (oh * p.stride_h - p.pad_h - win.ih_lo) * kWinW + ow * p.stride_w - p.pad_w + 4;
            win_valid = row < tile_rows(mt);
          }
        }
        if (win_base >= 0) {
          const bool valid = win_valid;
          const int base = win_base;
          const float* win_buf = windows + wb * (kWinBytes / 4);
#pragma unroll
          for (int j = 0; j < kBK / 4; ++j) {
            const int e = chunk_table[kb * (kBK / 4) + j];
            const int off = base + ((e >> 10) & 1023) * p.dil_h * kWinW + (e & 1023) * p.dil_w;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              v[4 * j + i] = (valid && e >= 0 && i < p.c) ? win_buf[i * kWinH * kWinW + off] : 0.0f;
            }
          }
        } else {
          const PixelSource px =
              pixel_source(x, p, row < tile_rows(tile / co_tiles) ? tile_p0(tile / co_tiles) + row : total_pixels,
                           total_pixels, pixels_per_image);
          gather_block(px, p, cp, kdim, plane, kb, chunk_table, v);
        }
        if (item + kGatherGroups >= last_end) mbar_arrive(&bars->win_empty[wb]);  // group's last item of the tile
        return true;
      }
      // The pixel's source row changes once per tile: 64-bit divisions only then.
      if (local != px_local) {
        px_local = local;
        px_cached = pixel_source(x, p, row < tile_rows(tile / co_tiles) ? tile_p0(tile / co_tiles) + row : total_pixels,
                                 total_pixels, pixels_per_image);
      }
      gather_block(px_cached, p, cp, kdim, plane, kb, use_table ? chunk_table : nullptr, v);
      return true;
    };
    // Splits one block into hi / lo and writes it to the stage's TMEM columns.
    // Returns false when the kernel is aborting.
    auto publish = [&](int item, float (&v)[kBK]) -> bool {
      if (CTB_TM_A_TMA) {
        // Activation ring: every item passes through it (a no-copy arrival
        // for items gathered from global memory) so its phases follow item.
        const int sa = item % kARing;
        if (!mbar_wait(&bars->a_full[sa], (item / kARing) & 1, abort, scratch, 40)) return false;
        int hw0, img;
        if (tile_a_tma(blockIdx.x + static_cast<long long>(item / k_blocks) * gridDim.x, &hw0, &img)) {
          const float* blk = a_ring + sa * kBK * kBM + row;
#pragma unroll
          for (int kk = 0; kk < kBK; ++kk) v[kk] = blk[kk * kBM];
        }
        mbar_arrive(&bars->a_empty[sa]);
      }
      const int s = item % kAStages;
      const int use = item / kAStages;
      if (use > 0 && !mbar_wait(&bars->empty_a[s], (use - 1) & 1, abort, scratch, 30)) return false;
      tc_fence_after_sync();
      const uint32_t a_col = tmem + lane_bits + T::kAColumn0 + s * 2 * kBK;
      uint32_t hi[kBK];
#pragma unroll
      for (int kk = 0; kk < kBK; ++kk) hi[kk] = __float_as_uint(v[kk]) & 0xFFFFE000u;
      tmem_store_32x32(a_col, hi);
      // lo = v - hi, in place (v is refilled by the next fetch).
#pragma unroll
      for (int kk = 0; kk < kBK; ++kk) v[kk] -= __uint_as_float(hi[kk]);
      tmem_store_32x32(a_col + kBK, reinterpret_cast<uint32_t(&)[kBK]>(v));
      tmem_store_wait();
      tc_fence_before_sync();
      mbar_arrive(&bars->full_a[s]);
      return true;
    };
    // Ping-pong register buffers: the group's next block is in flight while
    // the current one is split and stored (no register copy between them, so
    // nothing waits on the prefetch early).
    float buf_a[kBK], buf_b[kBK];
    int item = group;
    if (item < items && !fetch(item, buf_a)) item = items;
    while (item < items) {
      if (item + kGatherGroups < items && !fetch(item + kGatherGroups, buf_b)) break;
      if (!publish(item, buf_a)) break;
      item += kGatherGroups;
      if (item >= items) break;
      if (item + kGatherGroups < items && !fetch(item + kGatherGroups, buf_a)) break;
      if (!publish(item, buf_b)) break;
      item += kGatherGroups;
    }
  } else if (warp == 0 && lane == 0) {
    // ---- TMA producer: weight hi / lo tiles ----
    if (window_shape) tma_prefetch(tma_xwin);
    int g = 0;
    int windows_issued = 0;
    bool stop = false;
    // Window of tile L into buffer L % 2 once the gather groups have released
    // tile L - 2's. Tile L + 1's window is issued from the middle of tile L's
    // weight loop (block win_issue_block), so its copy lands before the gather
    // reaches it; issued with the tile's own weights it arrived late once per
    // tile. Waiting there for tile L - 1's release cannot stall: every copy
    // tile L - 1 needs is already issued.
    auto issue_window = [&](int L) -> bool {
      const int wb = L & 1;
      if (L >= 2 && !mbar_wait(&bars->win_empty[wb], ((L >> 1) - 1) & 1, abort, scratch, 44)) return false;
      const Window win = window_of(blockIdx.x + static_cast<long long>(L) * gridDim.x);
      if (win.ok) {
        mbar_arrive_expect_tx(&bars->win_full[wb], kWinBytes);
        tma_load_4d(windows + wb * (kWinBytes / 4), tma_xwin, &bars->win_full[wb], -4, win.ih_lo, 0, win.img);
      } else {
        mbar_arrive(&bars->win_full[wb]);
      }
      windows_issued = L + 1;
      return true;
    };
    const int win_issue_block = min(2, k_blocks - 1);
    for (int local = 0; local < my_tiles && !stop; ++local) {
      const long long tile = blockIdx.x + static_cast<long long>(local) * gridDim.x;
      const int co0 = static_cast<int>(tile % co_tiles) * BN;
      int a_hw0 = 0, a_img = 0;
      const bool tile_uses_a_tma = tile_a_tma(tile, &a_hw0, &a_img);
      if (window_shape && local == 0 && !issue_window(0)) break;
      for (int kb = 0; kb < k_blocks; ++kb, ++g) {
        const int s = g % kStages;
        const int use = g / kStages;
        if (use > 0 && !mbar_wait(&bars->empty_b[s], (use - 1) & 1, abort, scratch, 31)) {
          stop = true;
          break;
        }
        mbar_arrive_expect_tx(&bars->full_b[s], 2 * T::kPlaneBytes);
#pragma unroll
        for (int b = 0; b < BN / kBoxRows; ++b) {
          tma_load_3d(b_hi(s) + b * kBoxBytes, tma_w, &bars->full_b[s], kb * kBK, co0 + b * kBoxRows, 0);
          tma_load_3d(b_lo(s) + b * kBoxBytes, tma_w, &bars->full_b[s], kb * kBK, co0 + b * kBoxRows, 1);
        }
        if (CTB_TM_A_TMA) {
          const int sa = g % kARing;
          if (g >= kARing && !mbar_wait(&bars->a_empty[sa], (g / kARing - 1) & 1, abort, scratch, 41)) {
            stop = true;
            ++g;
            break;
          }
          if (tile_uses_a_tma) {
            mbar_arrive_expect_tx(&bars->a_full[sa], kBK * kBM * 4);
            tma_load_3d(a_ring + sa * kBK * kBM, tma_x, &bars->a_full[sa], a_hw0, kb * kBK, a_img);
          } else {
            mbar_arrive(&bars->a_full[sa]);
          }
        }
        if (window_shape && kb == win_issue_block && local + 1 < my_tiles && !issue_window(local + 1)) {
          stop = true;
          ++g;  // this block's weight copies are issued: the abort drain waits for them
          break;
        }
      }
    }
    if (*abort) {
      // Let every issued copy land before the CTA's shared memory is released.
      for (int q = *reinterpret_cast<volatile int*>(&bars->consumed); q < g; ++q) {
        volatile int never = 0;
        mbar_wait(&bars->full_b[q % kStages], (q / kStages) & 1, &never, scratch, 32);
      }
      if (window_shape) {
        // At most the two newest windows can still be in flight.
        for (int q = max(0, windows_issued - 2); q < windows_issued; ++q) {
          volatile int never = 0;
          mbar_wait(&bars->win_full[q & 1], (q >> 1) & 1, &never, scratch, 45);
        }
      }
      if (CTB_TM_A_TMA) {
        // At most one activation copy per ring slot can be outstanding.
        for (int q = max(0, g - kARing); q < g; ++q) {
          volatile int never = 0;
          mbar_wait(&bars->a_full[q % kARing], (q / kARing) & 1, &never, scratch, 42);
        }
      }
    }
  } else if (warp == 1 && lane == 0) {
    // ---- UMMA issuer ----
    constexpr uint32_t idesc = instr_desc(kFormatTF32, kBM, BN);  // A (TMEM) and B K-major
    int g = 0;
    bool ok = true;
    for (int local = 0; local < my_tiles && ok; ++local) {
      const int buf = local % T::kAccBufs;
      const int buf_use = local / T::kAccBufs;
      if (buf_use > 0 && !mbar_wait(&bars->tmem_empty[buf], (buf_use - 1) & 1, abort, scratch, 33)) {
        ok = false;
        break;
      }
      tc_fence_after_sync();
      const uint32_t acc = tmem + buf * T::kAccCols;
      for (int kb = 0; kb < k_blocks; ++kb, ++g) {
        const int s = g % kStages;   // weight stage
        const int sa = g % kAStages;  // activation stage
        if (!mbar_wait(&bars->full_b[s], (g / kStages) & 1, abort, scratch, 34) ||
            !mbar_wait(&bars->full_a[sa], (g / kAStages) & 1, abort, scratch, 35)) {
          ok = false;
          break;
        }
        tc_fence_after_sync();
        const uint64_t bhi = smem_desc_kmajor_sw128(b_hi(s));
        const uint64_t blo = smem_desc_kmajor_sw128(b_lo(s));
        const uint32_t ahi = tmem + T::kAColumn0 + sa * 2 * kBK;
        const uint32_t alo = ahi + kBK;
#pragma unroll
        for (int kk = 0; kk < kBK / 8; ++kk) {
          // 8 TF32 values along k: 8 TMEM columns of A, +32 bytes inside B's rows.
          const uint64_t dk = 2 * kk;
          if (T::kSplitN) {
            // [B_hi; B_lo] as one 128-row operand: b_lo(s) follows b_hi(s).
            constexpr uint32_t idesc_wide = instr_desc(kFormatTF32, kBM, 2 * BN);
            umma_tf32_ts(acc, ahi + 8 * kk, bhi + dk, idesc_wide, (kb | kk) != 0);
            umma_tf32_ts(acc, alo + 8 * kk, bhi + dk, idesc, 1);
          } else {
            umma_tf32_ts(acc, ahi + 8 * kk, bhi + dk, idesc, (kb | kk) != 0);
            umma_tf32_ts(acc, ahi + 8 * kk, blo + dk, idesc, 1);
            umma_tf32_ts(acc, alo + 8 * kk, bhi + dk, idesc, 1);
          }
        }
        umma_commit(&bars->empty_b[s]);
        umma_commit(&bars->empty_a[sa]);
        *reinterpret_cast<volatile int*>(&bars->consumed) = g + 1;
      }
      if (ok) umma_commit(&bars->tmem_full[buf]);
    }
    if (!ok) {
      umma_commit(&bars->drain);
      volatile int never = 0;
      mbar_wait(&bars->drain, 0, &never, scratch, 36);
    }
  } else if (warp >= kEpilogueWarp0 && warp < kEpilogueWarp0 + kEpiWarps) {
    // ---- epilogue: lane = output pixel, 32 channels per TMEM load ----
    const int quarter = warp & 3;                 // TMEM lanes this warp may access
    const int ew = (warp - kEpilogueWarp0) % 4;   // 0..3: which channel rows this warp copies
    const int half = (warp - kEpilogueWarp0) / 4;  // chunks ci with ci % kHalves == half
    constexpr int kChunks = BN / 32;
    // Folded BatchNorm terms of channel co0 + 32 i + lane, kept in registers
    // and broadcast with shuffles; reloaded only when the channel tile changes.
    float pm[kChunks], pa[kChunks], pb[kChunks];
    int prm_co0 = -1;
    auto load_params = [&](int co0) {
      if (kEpilogue == kPlain || co0 == prm_co0) return;
#pragma unroll
      for (int i = 0; i < kChunks; ++i) {
        const int co = co0 + 32 * i + lane;
        pm[i] = 0.0f;
        pa[i] = 0.0f;
        pb[i] = 0.0f;
        if (co < p.k) {
          pm[i] = mean[co];
          pa[i] = rsqrtf(variance[co] + epsilon) * scale[co];
          pb[i] = bias[co];
        }
      }
      prm_co0 = co0;
    };
    // BN affine, residual (from the staging slot) and ReLU of one chunk, in
    // place in v (lane = pixel). The slot reads all precede any store.
    auto finish_chunk = [&](int ci, const float* slot_px, uint32_t (&v)[32]) {
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        float x = __uint_as_float(v[j]);
        if (kEpilogue != kPlain) {
          x = (x - __shfl_sync(0xffffffffu, pm[ci], j)) * __shfl_sync(0xffffffffu, pa[ci], j) +
              __shfl_sync(0xffffffffu, pb[ci], j);
        }
        if (kEpilogue == kBatchNormAddRelu) x += slot_px[j * kBM];
        if (kEpilogue == kBatchNormRelu || kEpilogue == kBatchNormAddRelu) x = fmaxf(x, 0.0f);
        v[j] = __float_as_uint(x);
      }
    };
    auto tile_index = [&](int local) { return blockIdx.x + static_cast<long long>(local) * gridDim.x; };
    // Accumulator chunk ci (32 channels) of this warp's 32 rows.
    auto load_acc = [&](uint32_t taddr, int ci, uint32_t (&v)[32]) {
      tmem_load_32x32(taddr + 32 * ci, v);
      if (T::kSplitN) {
        uint32_t t[32];
        tmem_load_32x32(taddr + BN + 32 * ci, t);  // A_hi . B_lo
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = __float_as_uint(__uint_as_float(v[j]) + __uint_as_float(t[j]));
      }
    };

    if (bulk_epilogue) {
      // Bulk path: every 4-pixel group lies inside one image, so each channel
      // row of a tile is one or a few 16-byte-aligned runs in global memory.
      // Chunks (32 channels of a tile) go through a ring of kSlots staging
      // slots in shared memory ([32 channels][128 pixels] each). Chunk h: its
      // residual was bulk-loaded into slot h % kSlots four chunks earlier; the
      // result is written in place and leaves with one cp.async.bulk store per
      // run; then, once the store of chunk h - 2 has been read out, the
      // residual of chunk h + 4 is loaded into that slot. Lanes 0-7 of each
      // warp own channel row ew * 8 + lane of every chunk.
      const bool issuer = lane < 8;
      const int row = ew * 8 + lane;
      const int total_chunks = my_tiles * kChunks;
      // Calls fn(smem_offset_px, global_offset, pixels) for each run of
      // channel `ch` of tile `tile` (valid pixels only).
      auto for_each_run = [&](long long tile, int ch, auto&& fn) {
        const long long p0 = tile_p0(tile / co_tiles);
        const int n_valid = tile_rows(tile / co_tiles);
        long long img = p0 / pixels_per_image;
        int hw = static_cast<int>(p0 - img * pixels_per_image);
        for (int pos = 0; pos < n_valid; ++img, hw = 0) {
          const int len = min(n_valid - pos, static_cast<int>(pixels_per_image) - hw);
          fn(pos, (img * p.k + ch) * pixels_per_image + hw, len);
          pos += len;
        }
      };
      // A tile whose pixels lie in one image moves each chunk with a single
      // tensor copy: box {128 pixels, 32 channels, 1 image} of the [N][K][H*W]
      // view at (hw0, channel, image); pixels past H*W and channels past K are
      // clipped (stores) or zero-filled (loads). Tiles that straddle images
      // use one 1D copy per channel run.
      struct TileSpan {
        int hw0, img;
        bool one_image;
      };
      auto span_of = [&](long long tile) {
        const long long p0 = tile_p0(tile / co_tiles);
        const long long img = p0 / pixels_per_image;
        const int hw0 = static_cast<int>(p0 - img * pixels_per_image);
        const int n_valid = tile_rows(tile / co_tiles);
        return TileSpan{hw0, static_cast<int>(img), hw0 + n_valid <= pixels_per_image};
      };
      const bool leader = ew == 0 && lane == 0;  // issues the tensor copies
      auto load_residual = [&](int h) {
        if (kEpilogue != kBatchNormAddRelu || h >= total_chunks || !issuer) return;
        const int slot_id = h % kSlots;
        const long long tile = tile_index(h / kChunks);
        const int ch = static_cast<int>(tile % co_tiles) * BN + 32 * (h % kChunks) + row;
        float* slot_row = staging + (slot_id * 32 + row) * kBM;
        const TileSpan span = span_of(tile);
        if (span.one_image) {
          mbar_arrive_expect_tx(&bars->residual_full[slot_id], leader ? 32u * kBM * 4u : 0u);
          if (leader) {
            tma_load_3d(staging + slot_id * 32 * kBM, tma_res, &bars->residual_full[slot_id], span.hw0, ch - row,
                        span.img);
          }
          return;
        }
        uint32_t bytes = 0;
        if (ch < p.k) for_each_run(tile, ch, [&](int, long long, int len) { bytes += 4u * len; });
        mbar_arrive_expect_tx(&bars->residual_full[slot_id], bytes);
        if (ch < p.k) {
          for_each_run(tile, ch, [&](int pos, long long goff, int len) {
            asm volatile(
                "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                    smem_addr(slot_row + pos)),
                "l"(residual + goff), "r"(4 * len), "r"(smem_addr(&bars->residual_full[slot_id]))
                : "memory");
          });
        }
      };
#pragma unroll
      for (int h = 0; h < kLoadAhead; ++h) {
        if (h % kHalves == half) load_residual(h);
      }
      int local = 0;
      for (; local < my_tiles; ++local) {
        const int buf = local % T::kAccBufs;
        const long long tile = tile_index(local);
        const int co0 = static_cast<int>(tile % co_tiles) * BN;
        const TileSpan tile_span = span_of(tile);
        load_params(co0);
        const bool ready = mbar_wait(&bars->tmem_full[buf], (local / T::kAccBufs) & 1, abort, scratch, 37);
        // The four warps of a half leave together (they share named barriers).
        if (epilogue_any(half, !ready)) break;
        tc_fence_after_sync();
        const uint32_t taddr = tmem + buf * T::kAccCols + (static_cast<uint32_t>(quarter * 32) << 16);
#pragma unroll
        for (int ci = 0; ci < kChunks; ++ci) {
          if (ci % kHalves != half) continue;
          const int h = local * kChunks + ci;
          const int slot_id = h % kSlots;
          float* slot = staging + slot_id * 32 * kBM;
          if (kEpilogue == kBatchNormAddRelu) {
            // A timeout here is recorded (abort); the warps still walk the
            // same barrier sequence and leave at the next tile.
            mbar_wait(&bars->residual_full[slot_id], (h / kSlots) & 1, abort, scratch, 38);
          }
          uint32_t v[32];
          load_acc(taddr, ci, v);
          float* slot_px = slot + quarter * 32 + lane;
          finish_chunk(ci, slot_px, v);
#pragma unroll
          for (int j = 0; j < 32; ++j) slot_px[j * kBM] = __uint_as_float(v[j]);
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          epilogue_bar(half);  // the chunk is complete in shared memory
          if (issuer) {
            const int ch = co0 + 32 * ci + row;
            if (tile_span.one_image) {
              if (leader) {
                asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
                                 reinterpret_cast<uint64_t>(tma_out)),
                             "r"(smem_addr(slot)), "r"(tile_span.hw0), "r"(co0 + 32 * ci), "r"(tile_span.img)
                             : "memory");
              }
            } else if (ch < p.k) {
              for_each_run(tile, ch, [&](int pos, long long goff, int len) {
                asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(out + goff),
                             "r"(smem_addr(slot + row * kBM + pos)), "r"(4 * len)
                             : "memory");
              });
            }
            asm volatile("cp.async.bulk.commit_group;" ::: "memory");
            // This half's stores of chunks <= h + kLoadAhead - kSlots have been
            // read out of their slots.
            asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"((kSlots - kLoadAhead) / kHalves) : "memory");
          }
          epilogue_bar(half);
          load_residual(h + kLoadAhead);  // into slot (h + kLoadAhead - kSlots) % kSlots
        }
        // Hand the accumulator back to the issuer.
        tc_fence_before_sync();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars->tmem_empty[buf]);
      }
      if (issuer) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
      if (kEpilogue == kBatchNormAddRelu && issuer) {
        // Residual loads issued for chunks that were not reached (abort) must
        // land before the CTA's shared memory is released.
        const int consumed = local * kChunks;
        const int issued = min(total_chunks, consumed + kLoadAhead);
        for (int h = consumed; h < issued; ++h) {
          if (h % kHalves != half) continue;
          volatile int never = 0;
          mbar_wait(&bars->residual_full[h % kSlots], (h / kSlots) & 1, &never, scratch, 39);
        }
      }
    } else if (CTB_TM_A_TMA) {
      // 1x1 variant (even H and W): only misaligned output / residual pointers
      // come here. Plain loads and stores, kept small so the variant's common
      // path does not pay for this one in registers.
      for (int local = 0; local < my_tiles; ++local) {
        const int buf = local % T::kAccBufs;
        const long long tile = tile_index(local);
        const int co0 = static_cast<int>(tile % co_tiles) * BN;
        const long long pixel = tile_p0(tile / co_tiles) + quarter * 32 + lane;
        const bool valid = quarter * 32 + lane < tile_rows(tile / co_tiles);
        long long base = 0;
        if (valid) {
          const long long img = pixel / pixels_per_image;
          base = img * p.k * pixels_per_image + (pixel - img * pixels_per_image);
        }
        load_params(co0);
        const bool ready = mbar_wait(&bars->tmem_full[buf], (local / T::kAccBufs) & 1, abort, scratch, 37);
        if (epilogue_any(half, !ready)) break;
        tc_fence_after_sync();
        const uint32_t taddr = tmem + buf * T::kAccCols + (static_cast<uint32_t>(quarter * 32) << 16);
#pragma unroll
        for (int ci = 0; ci < kChunks; ++ci) {
          if (ci % kHalves != half) continue;
          const int ch0 = co0 + 32 * ci;
          uint32_t v[32];
          load_acc(taddr, ci, v);
          const int rows = min(32, p.k - ch0);
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            float x = __uint_as_float(v[j]);
            if (kEpilogue != kPlain) {
              x = (x - __shfl_sync(0xffffffffu, pm[ci], j)) * __shfl_sync(0xffffffffu, pa[ci], j) +
                  __shfl_sync(0xffffffffu, pb[ci], j);
            }
            const long long at = base + static_cast<long long>(ch0 + j) * pixels_per_image;
            if (kEpilogue == kBatchNormAddRelu && valid && j < rows) x += __ldg(residual + at);
            if (kEpilogue == kBatchNormRelu || kEpilogue == kBatchNormAddRelu) x = fmaxf(x, 0.0f);
            if (valid && j < rows) out[at] = x;
          }
        }
        tc_fence_before_sync();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars->tmem_empty[buf]);
      }
    } else {
      // Register path (pixels per image not a multiple of 4): residual
      // copied with 4-byte cp.async into the staging slots one tile ahead
      // (slot ci = chunk ci as [32 channels][128 pixels], channel rows split
      // over the four warps), results stored straight from registers.
      auto prefetch_residual = [&](int local, int ci) {
        if (kEpilogue != kBatchNormAddRelu) return;
        if (local < my_tiles) {
          const long long tile = tile_index(local);
          const int ch_base = static_cast<int>(tile % co_tiles) * BN + 32 * ci;
          const long long p0 = tile_p0(tile / co_tiles);
          const int rows = tile_rows(tile / co_tiles);
          float* slot = staging + ci * 32 * kBM;
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const long long px = p0 + 32 * q + lane;
            const bool pix_ok = 32 * q + lane < rows;
            long long src0 = 0;
            if (pix_ok) {
              const long long img = px / pixels_per_image;
              src0 = img * p.k * pixels_per_image + (px - img * pixels_per_image);
            }
#pragma unroll
            for (int j = ew; j < 32; j += 4) {
              const bool in = pix_ok && ch_base + j < p.k;
              const float* src = in ? residual + src0 + static_cast<long long>(ch_base + j) * pixels_per_image
                                    : residual;
              asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(
                               smem_addr(slot + j * kBM + 32 * q + lane)),
                           "l"(src), "r"(in ? 4 : 0)
                           : "memory");
            }
          }
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
      };
#pragma unroll
      for (int ci = 0; ci < kChunks; ++ci) prefetch_residual(0, ci);
      for (int local = 0; local < my_tiles; ++local) {
        const int buf = local % T::kAccBufs;
        const long long tile = tile_index(local);
        const int co0 = static_cast<int>(tile % co_tiles) * BN;
        const long long pixel = tile_p0(tile / co_tiles) + quarter * 32 + lane;
        const bool valid = quarter * 32 + lane < tile_rows(tile / co_tiles);
        long long base = 0;  // output offset of (image, channel 0, pixel)
        if (valid) {
          const long long img = pixel / pixels_per_image;
          base = img * p.k * pixels_per_image + (pixel - img * pixels_per_image);
        }
        load_params(co0);
        const bool ready = mbar_wait(&bars->tmem_full[buf], (local / T::kAccBufs) & 1, abort, scratch, 37);
        if (epilogue_any(half, !ready)) break;
        tc_fence_after_sync();
        const uint32_t taddr = tmem + buf * T::kAccCols + (static_cast<uint32_t>(quarter * 32) << 16);
#pragma unroll
        for (int ci = 0; ci < kChunks; ++ci) {
          const int ch0 = co0 + 32 * ci;
          if (kEpilogue == kBatchNormAddRelu) {
            asm volatile("cp.async.wait_group %0;" ::"n"(kChunks - 1) : "memory");
            epilogue_bar(half);  // every warp's part of chunk ci has landed
          }
          uint32_t v[32];
          load_acc(taddr, ci, v);
          finish_chunk(ci, staging + ci * 32 * kBM + quarter * 32 + lane, v);
          if (kEpilogue == kBatchNormAddRelu) {
            epilogue_bar(half);  // slot ci is free: refill it for the next tile
            prefetch_residual(local + 1, ci);
          }
          const int rows = min(32, p.k - ch0);
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            if (valid && j < rows) {
              out[base + static_cast<long long>(ch0 + j) * pixels_per_image] = __uint_as_float(v[j]);
            }
          }
        }
        tc_fence_before_sync();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars->tmem_empty[buf]);
      }
      // No copy may still be landing in shared memory when the CTA exits.
      if (kEpilogue == kBatchNormAddRelu) asm volatile("cp.async.wait_all;" ::: "memory");
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
__device__ __forceinline__ void conv_tm_dispatch(const TmaDescriptor* tma_w, const TmaDescriptor* tma_out,
                                                 const TmaDescriptor* tma_res, const TmaDescriptor* tma_x,
                                                 const TmaDescriptor* tma_xwin, const float* x, const float* scale,
                                                 const float* bias, const float* mean, const float* variance,
                                                 const float* residual, float* out, const ConvShape& p,
                                                 float epsilon, void* scratch) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
  if (p.k <= 64) {
    conv_tm<kEpilogue, 64>(smem, tma_w, tma_out, tma_res, tma_x, tma_xwin, x, scale, bias, mean, variance, residual, out, p, epsilon, scratch);
  } else {
    conv_tm<kEpilogue, 128>(smem, tma_w, tma_out, tma_res, tma_x, tma_xwin, x, scale, bias, mean, variance, residual, out, p, epsilon, scratch);
  }
}

}  // namespace

#define CTB_CONV_DIMS                                                                                 \
  int n, int c, int h, int w, int k, int r, int s, int out_h, int out_w, int stride_h, int stride_w, \
      int pad_h, int pad_w, int dilation_h, int dilation_w
#define CTB_CONV_SHAPE \
  ConvShape{n, c, h, w, k, r, s, out_h, out_w, stride_h, stride_w, pad_h, pad_w, dilation_h, dilation_w}

extern "C" __global__ void __launch_bounds__(kThreads, 1)
ctb_conv_f32_tm(const __grid_constant__ TmaDescriptor tma_w, const __grid_constant__ TmaDescriptor tma_out,
                const __grid_constant__ TmaDescriptor tma_x, const float* x, float* output, CTB_CONV_DIMS,
                CTB_RESERVED_PARAMS) {
  (void)profile_scratch;
  conv_tm_dispatch<kPlain>(&tma_w, &tma_out, nullptr, &tma_x, nullptr, x, nullptr, nullptr, nullptr, nullptr, nullptr, output, CTB_CONV_SHAPE, 0.0f,
                           runtime_scratch);
}

extern "C" __global__ void __launch_bounds__(kThreads, 1)
ctb_conv_bn_f32_tm(const __grid_constant__ TmaDescriptor tma_w, const __grid_constant__ TmaDescriptor tma_out,
                   const __grid_constant__ TmaDescriptor tma_x, const float* x, const float* scale, const float* bias, const float* mean, const float* variance,
                   float* output, CTB_CONV_DIMS, float epsilon, CTB_RESERVED_PARAMS) {
  (void)profile_scratch;
  conv_tm_dispatch<kBatchNorm>(&tma_w, &tma_out, nullptr, &tma_x, nullptr, x, scale, bias, mean, variance, nullptr, output, CTB_CONV_SHAPE, epsilon,
                               runtime_scratch);
}

extern "C" __global__ void __launch_bounds__(kThreads, 1)
ctb_conv_bn_relu_f32_tm(const __grid_constant__ TmaDescriptor tma_w, const __grid_constant__ TmaDescriptor tma_out,
                        const __grid_constant__ TmaDescriptor tma_x, const __grid_constant__ TmaDescriptor tma_xwin,
                        const float* x, const float* scale, const float* bias, const float* mean,
                        const float* variance, float* output, CTB_CONV_DIMS, float epsilon, CTB_RESERVED_PARAMS) {
  (void)profile_scratch;
  conv_tm_dispatch<kBatchNormRelu>(&tma_w, &tma_out, nullptr, &tma_x, &tma_xwin, x, scale, bias, mean, variance, nullptr, output, CTB_CONV_SHAPE,
                                   epsilon, runtime_scratch);
}

extern "C" __global__ void __launch_bounds__(kThreads, 1)
ctb_conv_bn_add_relu_f32_tm(const __grid_constant__ TmaDescriptor tma_w,
                            const __grid_constant__ TmaDescriptor tma_out,
                            const __grid_constant__ TmaDescriptor tma_res,
                            const __grid_constant__ TmaDescriptor tma_x, const float* x, const float* scale,
                            const float* bias, const float* mean, const float* variance, const float* residual,
                            float* output, CTB_CONV_DIMS, float epsilon, CTB_RESERVED_PARAMS) {
  (void)profile_scratch;
  conv_tm_dispatch<kBatchNormAddRelu>(&tma_w, &tma_out, &tma_res, &tma_x, nullptr, x, scale, bias, mean, variance, residual, output, CTB_CONV_SHAPE,
                                      epsilon, runtime_scratch);
}
