// Persistent FP16 GEMM / GEMM+GELU on CTA pairs (tcgen05 cta_group::2).
//
// C[M,N] = A[M,K] . B[K,N] (FP16 in, FP32 accumulate in TMEM, optional
// erf-GELU, round-to-nearest FP16 out): the math of
// python/cutriton/triton_kernels/transformer.py:17-107, like gemm_f16_tp.cu,
// with B prepacked once to B^T [N, K] ("transpose_2d").
//
// Two CTAs of a cluster (two SMs) share one 256 x BN output tile: CTA rank r
// holds rows 128 r .. 128 r + 127 of A and of the accumulator, and rows
// (BN / 2) r .. (BN / 2) r + BN / 2 - 1 of B^T; one tcgen05.mma.cta_group::2
// (M = 256, N = BN, K = 16) issued by the leader (rank 0) reads A and B from
// both CTAs' shared memory and accumulates into both CTAs' TMEM. Each SM
// therefore loads only half of B per k block: a 32 KB stage instead of
// 48 KB for BN = 256, six stages in flight instead of four.
//
// Pipeline (per CTA, 18 warps):
//   warp 0 lane 0 — TMA producer of this CTA's halves. Both CTAs' copies
//       complete on the leader's full barrier (the 2-CTA copy form, given the
//       leader's barrier by its cluster address); the leader's producer
//       announces the bytes of both. Each producer refills a stage after its
//       own empty barrier, which the leader's MMA commits arrive on in both
//       CTAs (one commit per CTA's barrier).
//   warp 1 lane 0 (leader only) — MMA issuer; its accumulator commits also
//       go to both CTAs.
//   warps 2-17 — epilogue of this CTA's 128 rows, as in gemm_f16_tp.cu; the
//       accumulator goes back to the issuer when all 32 epilogue warps of the
//       pair have read their columns (the peer's arrive remotely on the
//       leader's barrier).
// Every copy reads global memory into its own CTA's shared memory; nothing is
// broadcast across the cluster. All waits are bounded (tc_common.cuh).

#include "tc_common.cuh"

namespace {

using namespace ctb::tc;

constexpr int kBM = 128;  // rows per CTA (the pair covers 256)
constexpr int kBK = 64;
constexpr int kEpilogueWarps = 16;
constexpr int kThreads = (2 + kEpilogueWarps) * 32;
constexpr int kChunk = 32;
constexpr int kEpilogueWarp0 = 2;
constexpr uint32_t kTileA = kBM * kBK * 2;        // 16 KB
constexpr uint32_t kRingBytes = 196608;            // 6 x 32 KB
constexpr uint32_t kStageBoxBytes = 32 * kChunk * 2;
constexpr uint32_t kStagingBytes = kEpilogueWarps * kStageBoxBytes;
constexpr int kMaxStages = 8;

template <int BN>
struct Pair {
  static constexpr int kHalfB = BN / 2;  // B^T rows per CTA
  static constexpr uint32_t kTileB = kHalfB * kBK * 2;
  static constexpr uint32_t kStageBytes = kTileA + 16384;  // B slot sized for the widest half (128 rows)
  static constexpr int kStages = kRingBytes / kStageBytes;
  static_assert(kStages <= kMaxStages, "stage count");
  static constexpr uint32_t kTmemCols = (2 * BN) & (2 * BN - 1) ? 512 : 2 * BN;
  static constexpr int kChunks = BN / kChunk;
  static_assert(BN % kChunk == 0 && kChunks >= kEpilogueWarps / 4, "every epilogue warp takes a chunk");
};

struct __align__(8) Barriers {
  uint64_t full[kMaxStages];   // leader: both CTAs' copies of a stage landed
  uint64_t empty[kMaxStages];  // each CTA: the stage's MMAs are done
  uint64_t tmem_full[2];       // each CTA: the accumulator is complete
  uint64_t tmem_empty[2];      // leader: all 32 epilogue warps of the pair read it
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
  int consumed;
};

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// shared::cluster address of `local`'s counterpart in CTA `rank` of the pair.
__device__ __forceinline__ uint32_t cluster_addr(const void* local, uint32_t rank) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(smem_addr(local)), "r"(rank));
  return remote;
}

// 2D tile load into this CTA's shared memory whose completion counts on the
// barrier at `leader_bar` (a shared::cluster address in the pair leader).
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const TmaDescriptor* desc, uint32_t leader_bar, int x,
                                                 int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], "
      "[%2];" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(desc)), "r"(leader_bar), "r"(x), "r"(y)
      : "memory");
}

// Arrives once on `bar` in both CTAs when this thread's earlier MMAs are
// done: one commit to the local barrier, one to the peer's at the same
// offset (its shared::cluster address, rank 1).
__device__ __forceinline__ void umma_commit_pair(uint64_t* bar) {
  const uint32_t peer = cluster_addr(bar, 1);
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
               : "memory");
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(peer) : "memory");
}

__device__ __forceinline__ void umma_f16_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                              uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on the barrier at the same offset in the pair leader's shared memory.
__device__ __forceinline__ void arrive_on_leader(uint64_t* bar) {
  const uint32_t remote = cluster_addr(bar, 0);
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(remote) : "memory");
}

__device__ __forceinline__ void tma_store_2d(const TmaDescriptor* desc, const void* src, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(desc)),
               "r"(smem_addr(src)), "r"(x), "r"(y)
               : "memory");
}

template <bool kGelu, int BN>
__device__ __forceinline__ void gemm_pair(uint8_t* smem, const TmaDescriptor* tma_a, const TmaDescriptor* tma_b,
                                          const TmaDescriptor* tma_out, __half* out, int m, int n, int k,
                                          void* scratch) {
  using P = Pair<BN>;
  constexpr int kStages = P::kStages;
  uint8_t* staging = smem + kRingBytes;
  Barriers* bars = reinterpret_cast<Barriers*>(staging + kStagingBytes);
  volatile int* abort = &bars->abort;
  auto tile_a = [&](int s) { return smem + s * P::kStageBytes; };
  auto tile_b = [&](int s) { return smem + s * P::kStageBytes + kTileA; };

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const bool leader = rank == 0;
  const int pairs = gridDim.x / 2;
  const int pair = blockIdx.x / 2;
  const int k_blocks = (k + kBK - 1) / kBK;
  const int n_tiles = (n + BN - 1) / BN;
  const int tiles = ((m + 2 * kBM - 1) / (2 * kBM)) * n_tiles;
  const int my_tiles = tiles > pair ? (tiles - 1 - pair) / pairs + 1 : 0;
  const bool tma_epilogue = n % 8 == 0 && (reinterpret_cast<uintptr_t>(out) & 15) == 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bars->full[s], 1);
      mbar_init(&bars->empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&bars->tmem_full[b], 1);
      mbar_init(&bars->tmem_empty[b], 2 * kEpilogueWarps);
    }
    mbar_init(&bars->drain, 1);
    bars->abort = 0;
    bars->consumed = 0;
    mbar_init_fence();
    tma_prefetch(tma_a);
    tma_prefetch(tma_b);
    if (tma_epilogue) tma_prefetch(tma_out);
  }
  // The peer's copies and commits reach these barriers: both CTAs have
  // initialised them before either goes on.
  cluster_sync();
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(&bars->tmem_base)),
                 "r"(P::kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  const uint32_t tmem = bars->tmem_base;
  CTB_GRID_DEPENDENCY_SYNC();

  if (warp == 0 && lane == 0) {
    // ---- TMA producer: this CTA's A rows and B^T rows ----
    int g = 0;
    bool stop = false;
    for (int local = 0; local < my_tiles && !stop; ++local) {
      const int tile = pair + local * pairs;
      const int m0 = (tile / n_tiles) * 2 * kBM + static_cast<int>(rank) * kBM;
      const int n0 = (tile % n_tiles) * BN + static_cast<int>(rank) * P::kHalfB;
      for (int kb = 0; kb < k_blocks; ++kb, ++g) {
        const int s = g % kStages;
        const int use = g / kStages;
        if (use > 0 && !mbar_wait(&bars->empty[s], (use - 1) & 1, abort, scratch, 60)) {
          stop = true;
          break;
        }
        if (leader) mbar_arrive_expect_tx(&bars->full[s], 2 * (kTileA + P::kTileB));
        const uint32_t full_on_leader = cluster_addr(&bars->full[s], 0);
        tma_load_2d_pair(tile_a(s), tma_a, full_on_leader, kb * kBK, m0);
        tma_load_2d_pair(tile_b(s), tma_b, full_on_leader, kb * kBK, n0);
      }
    }
    if (*abort && leader) {
      // Let the issued copies land before shared memory is released (the
      // peer's too: the leader's barrier counts them). Bounded: a phase the
      // aborted peer never fed times out after the wait limit.
      for (int q = *reinterpret_cast<volatile int*>(&bars->consumed); q < g; ++q) {
        volatile int never = 0;
        mbar_wait(&bars->full[q % kStages], (q / kStages) & 1, &never, scratch, 61);
      }
    }
  } else if (warp == 1 && lane == 0 && leader) {
    // ---- MMA issuer (pair leader) ----
    constexpr uint32_t idesc = instr_desc(kFormatF16, 2 * kBM, BN);
    int g = 0;
    bool ok = true;
    for (int local = 0; local < my_tiles && ok; ++local) {
      const int buf = local & 1;
      if (local >= 2 && !mbar_wait(&bars->tmem_empty[buf], ((local >> 1) - 1) & 1, abort, scratch, 62)) {
        ok = false;
        break;
      }
      tc_fence_after_sync();
      const uint32_t acc = tmem + buf * BN;
      for (int kb = 0; kb < k_blocks; ++kb, ++g) {
        const int s = g % kStages;
        if (!mbar_wait(&bars->full[s], (g / kStages) & 1, abort, scratch, 63)) {
          ok = false;
          break;
        }
        tc_fence_after_sync();
        const uint64_t a_desc = smem_desc_kmajor_sw128(tile_a(s));
        const uint64_t b_desc = smem_desc_kmajor_sw128(tile_b(s));
#pragma unroll
        for (int kk = 0; kk < kBK / 16; ++kk) {
          umma_f16_pair(acc, a_desc + 2 * kk, b_desc + 2 * kk, idesc, (kb | kk) != 0);
        }
        umma_commit_pair(&bars->empty[s]);
        *reinterpret_cast<volatile int*>(&bars->consumed) = g + 1;
      }
      if (ok) umma_commit_pair(&bars->tmem_full[buf]);
    }
    if (!ok) {
      asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                       smem_addr(&bars->drain))
                   : "memory");
      volatile int never = 0;
      mbar_wait(&bars->drain, 0, &never, scratch, 64);
    }
  } else if (warp >= kEpilogueWarp0) {
    // ---- epilogue: this CTA's 128 rows, quarter = warp % 4 ----
    constexpr int kPacks = kChunk / 8;
    constexpr int kWarpsPerQuarter = kEpilogueWarps / 4;
    const int quarter = warp & 3;
    const int wq = (warp - kEpilogueWarp0) / 4;
    uint8_t* box = staging + (warp - kEpilogueWarp0) * kStageBoxBytes;
    bool box_used = false;
    for (int local = 0; local < my_tiles; ++local) {
      const int buf = local & 1;
      const int tile = pair + local * pairs;
      const int m0 = (tile / n_tiles) * 2 * kBM + static_cast<int>(rank) * kBM;
      const int n0 = (tile % n_tiles) * BN;
      const bool ready = mbar_wait(&bars->tmem_full[buf], (local >> 1) & 1, abort, scratch, 65);
      __syncwarp();
      if (!ready) break;
      tc_fence_after_sync();
      const uint32_t taddr = tmem + buf * BN + (static_cast<uint32_t>(quarter * 32) << 16);
      const int row = m0 + quarter * 32 + lane;
#pragma unroll 1
      for (int ci = wq; ci < P::kChunks; ci += kWarpsPerQuarter) {
        const int c = ci * kChunk;
        uint32_t v[kChunk];
        tmem_load_32x32(taddr + c, v);
        if (ci + kWarpsPerQuarter >= P::kChunks) {
          // This warp's columns are in registers: release them to the issuer.
          tc_fence_before_sync();
          __syncwarp();
          if (lane == 0) {
            if (leader) {
              mbar_arrive(&bars->tmem_empty[buf]);
            } else {
              arrive_on_leader(&bars->tmem_empty[buf]);
            }
          }
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
  // Neither CTA leaves (or frees TMEM) while its peer may still signal it.
  cluster_sync();
  tc_fence_after_sync();
  if (warp == 0) {
    __syncwarp();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(P::kTmemCols) : "memory");
  }
}

template <bool kGelu>
__device__ __forceinline__ void gemm_pair_dispatch(const TmaDescriptor* tma_a, const TmaDescriptor* tma_b128,
                                                   const TmaDescriptor* tma_b96, const TmaDescriptor* tma_b64,
                                                   const TmaDescriptor* tma_out, __half* out, int m, int n, int k,
                                                   void* scratch) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
  // Pair tiles are 256 x BN; the same waves x tile-cost rule as the
  // single-CTA kernel, over pairs of SMs. Both CTAs of a pair compute it
  // from the same inputs, so they agree.
  const long long m_tiles = (m + 2 * kBM - 1) / (2 * kBM);
  const long long g = gridDim.x / 2;
  const long long w256 = (m_tiles * ((n + 255) / 256) + g - 1) / g;
  const long long w192 = (m_tiles * ((n + 191) / 192) + g - 1) / g;
  const long long w128 = (m_tiles * ((n + 127) / 128) + g - 1) / g;
  const long long t256 = 100 * w256, t192 = 80 * w192, t128 = 69 * w128;
  if (t256 <= t192 && t256 <= t128) {
    gemm_pair<kGelu, 256>(smem, tma_a, tma_b128, tma_out, out, m, n, k, scratch);
  } else if (t192 <= t128) {
    gemm_pair<kGelu, 192>(smem, tma_a, tma_b96, tma_out, out, m, n, k, scratch);
  } else {
    gemm_pair<kGelu, 128>(smem, tma_a, tma_b64, tma_out, out, m, n, k, scratch);
  }
}

}  // namespace

// B^T arrives through one of three maps whose boxes are the half-tile row
// counts of the three tile widths (128, 96, 64 rows).
extern "C" __global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
ctb_gemm_f16_2sm(const __grid_constant__ TmaDescriptor tma_a, const __grid_constant__ TmaDescriptor tma_b128,
                 const __grid_constant__ TmaDescriptor tma_b96, const __grid_constant__ TmaDescriptor tma_b64,
                 const __grid_constant__ TmaDescriptor tma_out, __half* output, int m, int n, int k,
                 CTB_RESERVED_PARAMS) {
  (void)profile_scratch;
  gemm_pair_dispatch<false>(&tma_a, &tma_b128, &tma_b96, &tma_b64, &tma_out, output, m, n, k, runtime_scratch);
}

extern "C" __global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
ctb_gemm_gelu_f16_2sm(const __grid_constant__ TmaDescriptor tma_a, const __grid_constant__ TmaDescriptor tma_b128,
                      const __grid_constant__ TmaDescriptor tma_b96, const __grid_constant__ TmaDescriptor tma_b64,
                      const __grid_constant__ TmaDescriptor tma_out, __half* output, int m, int n, int k,
                      CTB_RESERVED_PARAMS) {
  (void)profile_scratch;
  gemm_pair_dispatch<true>(&tma_a, &tma_b128, &tma_b96, &tma_b64, &tma_out, output, m, n, k, runtime_scratch);
}
