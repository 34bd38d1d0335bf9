// Persistent FP16 GEMM / GEMM+GELU on the 5th-generation tensor cores.
//
// C[M,N] = A[M,K] . B[K,N] (FP16 in, FP32 accumulate in TMEM, optional
// erf-GELU (erf to 1.5e-7, common.cuh), round-to-nearest FP16 out) — the math of
// python/cutriton/triton_kernels/transformer.py:17-107. B is a constant
// weight prepacked once to B^T [N, K] ("transpose_2d"), so both operands are
// K-major and staged by TMA in the 128-byte-swizzled layout the UMMA
// descriptors read.
//
// One CTA per SM walks the 128 x BN output tiles (BN = 256, 192 or 128,
// whichever gives the fewest estimated waves x tile cost) in a static
// round-robin, N fastest so co-running CTAs share the A tile in L2. Roles
// (18 warps):
//   warp 0 lane 0 — TMA producer: A (128 x 64) and B (BN x 64) per k block
//       through a STAGES-deep shared-memory ring (full / empty barriers);
//   warp 1 lane 0 — UMMA issuer: 4 x (128 x BN x 16) per k block into one of
//       two TMEM accumulators (2 x BN columns), so the epilogue of one tile
//       overlaps the MMAs of the next;
//   warps 2-17 — epilogue, four warps per TMEM lane quarter (warp % 4 = 32
//       rows), taking the quarter's 32-column chunks in turn -> GELU ->
//       FP16 -> a 32 x 32 staging box in shared memory (64-byte swizzle,
//       conflict-free 16-byte writes) -> TMA tensor store; each warp hands its
//       columns of the accumulator back as soon as they are in registers.
//       The erf-GELU is latency-bound (two MUFU ops in a dependent chain per
//       element): sixteen warps, four per scheduler, hide it where eight
//       left the epilogue of a tile longer than the next tile's MMAs.
// All waits are bounded (tc_common.cuh).

#include "tc_common.cuh"

namespace {

using namespace ctb::tc;

constexpr int kBM = 128;
constexpr int kBK = 64;  // FP16 elements per 128-byte swizzle row
constexpr int kEpilogueWarps = 16;
constexpr int kThreads = (2 + kEpilogueWarps) * 32;
// Columns per staging chunk: 32 FP16 = 64-byte rows, stored through a
// 64-byte-swizzled 32 x 32 TMA box.
constexpr int kChunk = 32;
constexpr int kEpilogueWarp0 = 2;
constexpr uint32_t kTileA = kBM * kBK * 2;      // 16 KB
constexpr uint32_t kBoxRowsB = 128;              // B rows (N) per TMA box
constexpr uint32_t kRingBytes = 196608;          // 4 x (16 + 32) KB = 6 x (16 + 16) KB
constexpr uint32_t kStageBoxBytes = 32 * kChunk * 2;  // 2 KB: 32 rows x 32 FP16
constexpr uint32_t kStagingBytes = kEpilogueWarps * kStageBoxBytes;
constexpr int kMaxStages = 6;

template <int BN>
struct Config {
  // B arrives in 128-row boxes: a 192-wide tile loads two (the last 64 rows
  // unused), so its stage is as large as a 256-wide one's.
  static constexpr int kBoxesB = (BN + kBoxRowsB - 1) / kBoxRowsB;
  static constexpr int kStages = BN == 128 ? 6 : 4;
  static constexpr uint32_t kTileB = kBoxesB * kBoxRowsB * kBK * 2;
  static constexpr uint32_t kStageBytes = kTileA + kTileB;
  static_assert(kStages * kStageBytes <= kRingBytes, "shared memory ring");
  static_assert(2 * BN <= 512, "TMEM accumulators");
  // Two accumulators of BN columns; allocations are powers of two.
  static constexpr uint32_t kTmemCols = (2 * BN) & (2 * BN - 1) ? 512 : 2 * BN;
  static constexpr int kChunks = BN / kChunk;  // 32-column epilogue chunks per lane quarter
  static_assert(BN % kChunk == 0 && kChunks >= kEpilogueWarps / 4, "every epilogue warp takes a chunk");
};

struct __align__(8) Barriers {
  uint64_t full[kMaxStages];
  uint64_t empty[kMaxStages];
  uint64_t tmem_full[2];
  uint64_t tmem_empty[2];
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
  int consumed;
};

__device__ __forceinline__ void tma_store_2d(const TmaDescriptor* desc, const void* src, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(desc)),
               "r"(smem_addr(src)), "r"(x), "r"(y)
               : "memory");
}

template <bool kGelu, int BN>
__device__ __forceinline__ void gemm_tp(uint8_t* smem, const TmaDescriptor* tma_a, const TmaDescriptor* tma_b,
                                        const TmaDescriptor* tma_out, __half* out, int m, int n, int k,
                                        void* scratch) {
  using C = Config<BN>;
  constexpr int kStages = C::kStages;
  uint8_t* staging = smem + kRingBytes;
  Barriers* bars = reinterpret_cast<Barriers*>(staging + kStagingBytes);
  volatile int* abort = &bars->abort;
  auto tile_a = [&](int s) { return smem + s * C::kStageBytes; };
  auto tile_b = [&](int s) { return smem + s * C::kStageBytes + kTileA; };

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  const int k_blocks = (k + kBK - 1) / kBK;
  const int n_tiles = (n + BN - 1) / BN;
  const int tiles = ((m + kBM - 1) / kBM) * n_tiles;
  const int my_tiles = tiles > static_cast<int>(blockIdx.x) ? (tiles - 1 - blockIdx.x) / gridDim.x + 1 : 0;
  // TMA stores need 16-byte aligned rows; tma_out is bound as zeros otherwise.
  const bool tma_epilogue = n % 8 == 0 && (reinterpret_cast<uintptr_t>(out) & 15) == 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bars->full[s], 1);
      mbar_init(&bars->empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&bars->tmem_full[b], 1);
      mbar_init(&bars->tmem_empty[b], kEpilogueWarps);
    }
    mbar_init(&bars->drain, 1);
    bars->abort = 0;
    bars->consumed = 0;
    mbar_init_fence();
    tma_prefetch(tma_a);
    tma_prefetch(tma_b);
    if (tma_epilogue) tma_prefetch(tma_out);
  }
  if (warp == 0) tmem_alloc(&bars->tmem_base, C::kTmemCols);
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  const uint32_t tmem = bars->tmem_base;
  // Activations are touched only after the preceding kernel has finished.
  CTB_GRID_DEPENDENCY_SYNC();

  if (warp == 0 && lane == 0) {
    // ---- TMA producer ----
    int g = 0;
    bool stop = false;
    for (int local = 0; local < my_tiles && !stop; ++local) {
      const int tile = blockIdx.x + local * gridDim.x;
      const int m0 = (tile / n_tiles) * kBM;
      const int n0 = (tile % n_tiles) * BN;
      for (int kb = 0; kb < k_blocks; ++kb, ++g) {
        const int s = g % kStages;
        const int use = g / kStages;
        if (use > 0 && !mbar_wait(&bars->empty[s], (use - 1) & 1, abort, scratch, 50)) {
          stop = true;
          break;
        }
        mbar_arrive_expect_tx(&bars->full[s], C::kStageBytes);
        tma_load_2d(tile_a(s), tma_a, &bars->full[s], kb * kBK, m0);
#pragma unroll
        for (int b = 0; b < C::kBoxesB; ++b) {
          tma_load_2d(tile_b(s) + b * kBoxRowsB * 128, tma_b, &bars->full[s], kb * kBK, n0 + b * kBoxRowsB);
        }
      }
    }
    if (*abort) {
      // Let every issued copy land before the CTA's shared memory is released.
      for (int q = *reinterpret_cast<volatile int*>(&bars->consumed); q < g; ++q) {
        volatile int never = 0;
        mbar_wait(&bars->full[q % kStages], (q / kStages) & 1, &never, scratch, 51);
      }
    }
  } else if (warp == 1 && lane == 0) {
    // ---- UMMA issuer ----
    constexpr uint32_t idesc = instr_desc(kFormatF16, kBM, BN);
    int g = 0;
    bool ok = true;
    for (int local = 0; local < my_tiles && ok; ++local) {
      const int buf = local & 1;
      if (local >= 2 && !mbar_wait(&bars->tmem_empty[buf], ((local >> 1) - 1) & 1, abort, scratch, 52)) {
        ok = false;
        break;
      }
      tc_fence_after_sync();
      const uint32_t acc = tmem + buf * BN;
      for (int kb = 0; kb < k_blocks; ++kb, ++g) {
        const int s = g % kStages;
        if (!mbar_wait(&bars->full[s], (g / kStages) & 1, abort, scratch, 53)) {
          ok = false;
          break;
        }
        tc_fence_after_sync();
        const uint64_t a_desc = smem_desc_kmajor_sw128(tile_a(s));
        const uint64_t b_desc = smem_desc_kmajor_sw128(tile_b(s));
#pragma unroll
        for (int kk = 0; kk < kBK / 16; ++kk) {
          // +32 bytes per 16-element K step inside the swizzled rows.
          umma_f16(acc, a_desc + 2 * kk, b_desc + 2 * kk, idesc, (kb | kk) != 0);
        }
        umma_commit(&bars->empty[s]);
        *reinterpret_cast<volatile int*>(&bars->consumed) = g + 1;
      }
      if (ok) umma_commit(&bars->tmem_full[buf]);
    }
    if (!ok) {
      umma_commit(&bars->drain);
      volatile int never = 0;
      mbar_wait(&bars->drain, 0, &never, scratch, 54);
    }
  } else if (warp >= kEpilogueWarp0) {
    // ---- epilogue: rows quarter*32 + lane; the quarter's 32-column chunks
    // are dealt round-robin to its four warps (chunk ci to warp ci % 4) ----
    constexpr int kPacks = kChunk / 8;
    constexpr int kWarpsPerQuarter = kEpilogueWarps / 4;
    const int quarter = warp & 3;
    const int wq = (warp - kEpilogueWarp0) / 4;  // this warp's rank within its quarter
    uint8_t* box = staging + (warp - kEpilogueWarp0) * kStageBoxBytes;
    bool box_used = false;
    for (int local = 0; local < my_tiles; ++local) {
      const int buf = local & 1;
      const int tile = blockIdx.x + local * gridDim.x;
      const int m0 = (tile / n_tiles) * kBM;
      const int n0 = (tile % n_tiles) * BN;
      const bool ready = mbar_wait(&bars->tmem_full[buf], (local >> 1) & 1, abort, scratch, 55);
      __syncwarp();
      if (!ready) break;
      tc_fence_after_sync();
      const uint32_t taddr = tmem + buf * BN + (static_cast<uint32_t>(quarter * 32) << 16);
      const int row = m0 + quarter * 32 + lane;
#pragma unroll 1
      for (int ci = wq; ci < C::kChunks; ci += kWarpsPerQuarter) {
        const int c = ci * kChunk;
        uint32_t v[kChunk];
        tmem_load_32x32(taddr + c, v);
        if (ci + kWarpsPerQuarter >= C::kChunks) {
          // This warp's columns of the accumulator are in registers: hand them back.
          tc_fence_before_sync();
          __syncwarp();
          if (lane == 0) mbar_arrive(&bars->tmem_empty[buf]);
        }
        uint4 packed[kPacks];
#pragma unroll
        for (int ch = 0; ch < kPacks; ++ch) {
          __half2* h = reinterpret_cast<__half2*>(&packed[ch]);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            float a = __uint_as_float(v[ch * 8 + 2 * j]);
            float b = __uint_as_float(v[ch * 8 + 2 * j + 1]);
            if (kGelu) {
              a = ctb::gelu_erf_fast(a);
              b = ctb::gelu_erf_fast(b);
            }
            h[j] = __floats2half2_rn(a, b);
          }
        }
        if (n0 + c >= n) {
          // Columns past N (a partial last tile): nothing to store.
        } else if (tma_epilogue) {
          if (box_used) {
            // The previous store from this box has read it out.
            if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
            __syncwarp();
          }
          // Row `lane` (64 bytes); 64-byte swizzle: 16-byte chunk j at j ^ ((lane / 2) % 4).
#pragma unroll
          for (int ch = 0; ch < kPacks; ++ch) {
            *reinterpret_cast<uint4*>(box + lane * 64 + (((ch ^ (lane >> 1)) & 3) << 4)) = packed[ch];
          }
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(tma_out, box, n0 + c, m0 + quarter * 32);
            asm volatile("cp.async.bulk.commit_group;" ::: "memory");
          }
          box_used = true;
        } else if (row < m) {
          __half* dst = out + static_cast<long long>(row) * n + n0 + c;
#pragma unroll
          for (int ch = 0; ch < kPacks; ++ch) {
            if (n0 + c + ch * 8 < n) *reinterpret_cast<uint4*>(dst + ch * 8) = packed[ch];
          }
        }
      }
    }
    if (lane == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
  }
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  if (warp == 0) {
    __syncwarp();
    tmem_dealloc(tmem, C::kTmemCols);
  }
}

template <bool kGelu>
__device__ __forceinline__ void gemm_tp_dispatch(const TmaDescriptor* tma_a, const TmaDescriptor* tma_b,
                                                 const TmaDescriptor* tma_out, __half* out, int m, int n, int k,
                                                 void* scratch) {
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte alignment for the 128-byte swizzle atoms.
  uint8_t* smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
  const long long m_tiles = (m + kBM - 1) / kBM;
  // Estimated time = waves x per-tile cost, relative to a 256-wide tile (100):
  // a 128-wide tile costs ~69 at steady state (measured), a 192-wide one ~80
  // (three quarters of the MMAs, two B boxes). 192 wins where 256-wide tiles
  // leave SMs idle, e.g. N = 768 at M = 4096: 96 tiles on 148 SMs.
  const long long g = gridDim.x;
  const long long w256 = (m_tiles * ((n + 255) / 256) + g - 1) / g;
  const long long w192 = (m_tiles * ((n + 191) / 192) + g - 1) / g;
  const long long w128 = (m_tiles * ((n + 127) / 128) + g - 1) / g;
  const long long t256 = 100 * w256, t192 = 80 * w192, t128 = 69 * w128;
  if (t256 <= t192 && t256 <= t128) {
    gemm_tp<kGelu, 256>(smem, tma_a, tma_b, tma_out, out, m, n, k, scratch);
  } else if (t192 <= t128) {
    gemm_tp<kGelu, 192>(smem, tma_a, tma_b, tma_out, out, m, n, k, scratch);
  } else {
    gemm_tp<kGelu, 128>(smem, tma_a, tma_b, tma_out, out, m, n, k, scratch);
  }
}

}  // namespace

extern "C" __global__ void __launch_bounds__(kThreads, 1)
ctb_gemm_f16_tp(const __grid_constant__ TmaDescriptor tma_a, const __grid_constant__ TmaDescriptor tma_b,
                const __grid_constant__ TmaDescriptor tma_out, __half* output, int m, int n, int k,
                CTB_RESERVED_PARAMS) {
  (void)profile_scratch;
  gemm_tp_dispatch<false>(&tma_a, &tma_b, &tma_out, output, m, n, k, runtime_scratch);
}

extern "C" __global__ void __launch_bounds__(kThreads, 1)
ctb_gemm_gelu_f16_tp(const __grid_constant__ TmaDescriptor tma_a, const __grid_constant__ TmaDescriptor tma_b,
                     const __grid_constant__ TmaDescriptor tma_out, __half* output, int m, int n, int k,
                     CTB_RESERVED_PARAMS) {
  (void)profile_scratch;
  gemm_tp_dispatch<true>(&tma_a, &tma_b, &tma_out, output, m, n, k, runtime_scratch);
}
