// FP16 GEMM / GEMM+GELU on the 5th-generation tensor cores (tcgen05).
//
// C[M,N] = A[M,K] . B[K,N] (FP16 in, FP32 accumulate in TMEM, optional
// exact-erf GELU on the accumulator, round-to-nearest FP16 out) — the math of
// python/cutriton/triton_kernels/transformer.py:17-107. B is a constant
// weight: the engine prepacks it once to B^T [N, K] ("transpose_2d"), so both
// operands are K-major and both are staged by TMA in the 128-byte-swizzled
// layout the UMMA descriptors read directly.
//
// One 128 x BN output tile per CTA, K in blocks of 64 (one 128-byte swizzle
// row of FP16) through a STAGES-deep TMA -> smem ring:
//   warp 0 lane 0: TMA producer (full[s] barriers, expect_tx bytes);
//   warp 1 lane 0: UMMA issuer, 4 x (128 x BN x 16) per k-block, commits
//                  empty[s] when the MMAs reading stage s retire;
//   warp 2:        allocates / frees the BN TMEM columns of the accumulator;
//   warps 0-3:     epilogue — TMEM lanes 32w..32w+31 (warp w's quarter) ->
//                  registers -> GELU -> FP16 -> 16-byte global stores.
// Compile-time BLOCK_N (128 or 256) and STAGES come from the pack variant.

#include "tc_common.cuh"

#ifndef CTB_BLOCK_N
#define CTB_BLOCK_N 128
#endif
#ifndef CTB_STAGES
#define CTB_STAGES 4
#endif

namespace {

using namespace ctb::tc;

constexpr int kBM = 128;
constexpr int kBN = CTB_BLOCK_N;
constexpr int kBK = 64;  // FP16 elements per 128-byte swizzle row
constexpr int kStages = CTB_STAGES;
constexpr int kThreads = 128;
constexpr uint32_t kTileA = kBM * kBK * 2;
constexpr uint32_t kTileB = kBN * kBK * 2;
constexpr uint32_t kTmemCols = kBN;  // FP32 accumulator: one column per N
static_assert(kBN == 128 || kBN == 256, "BLOCK_N must be 128 or 256");

struct __align__(8) Barriers {
  uint64_t full[kStages];
  uint64_t empty[kStages];
  uint64_t accum;
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
  int consumed;
};

template <bool kGelu>
__device__ __forceinline__ void gemm_tc(const TmaDescriptor* tma_a, const TmaDescriptor* tma_b, __half* out, int m,
                                        int n, int k, void* scratch) {
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte alignment for the 128-byte swizzle atoms.
  uint8_t* smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
  uint8_t* tiles_a = smem;
  uint8_t* tiles_b = smem + kStages * kTileA;
  Barriers* bars = reinterpret_cast<Barriers*>(tiles_b + kStages * kTileB);
  volatile int* abort = &bars->abort;

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  const int m0 = blockIdx.x * kBM;
  const int n0 = blockIdx.y * kBN;
  const int k_blocks = (k + kBK - 1) / kBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bars->full[s], 1);
      mbar_init(&bars->empty[s], 1);
    }
    mbar_init(&bars->accum, 1);
    mbar_init(&bars->drain, 1);
    bars->abort = 0;
    bars->consumed = 0;
    mbar_init_fence();
    tma_prefetch(tma_a);
    tma_prefetch(tma_b);
  }
  if (warp == 2) tmem_alloc(&bars->tmem_base, kTmemCols);
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  const uint32_t tmem = bars->tmem_base;
  // Activations are touched only after the preceding kernel has finished.
  CTB_GRID_DEPENDENCY_SYNC();

  if (warp == 0 && lane == 0) {
    // TMA producer.
    int issued = 0;
    for (int kb = 0; kb < k_blocks; ++kb) {
      const int s = kb % kStages;
      const int use = kb / kStages;
      if (use > 0 && !mbar_wait(&bars->empty[s], (use - 1) & 1, abort, scratch, 1)) break;
      mbar_arrive_expect_tx(&bars->full[s], kTileA + kTileB);
      tma_load_2d(tiles_a + s * kTileA, tma_a, &bars->full[s], kb * kBK, m0);
      tma_load_2d(tiles_b + s * kTileB, tma_b, &bars->full[s], kb * kBK, n0);
      issued = kb + 1;
    }
    if (*abort) {
      // Let every issued copy land before the CTA's smem is released.
      for (int kb = *reinterpret_cast<volatile int*>(&bars->consumed); kb < issued; ++kb) {
        volatile int never = 0;
        mbar_wait(&bars->full[kb % kStages], (kb / kStages) & 1, &never, scratch, 2);
      }
    }
  } else if (warp == 1 && lane == 0) {
    // UMMA issuer.
    constexpr uint32_t idesc = instr_desc(kFormatF16, kBM, kBN);
    bool ok = true;
    for (int kb = 0; kb < k_blocks; ++kb) {
      const int s = kb % kStages;
      if (!mbar_wait(&bars->full[s], (kb / kStages) & 1, abort, scratch, 3)) {
        ok = false;
        break;
      }
      tc_fence_after_sync();
      const uint64_t a_desc = smem_desc_kmajor_sw128(tiles_a + s * kTileA);
      const uint64_t b_desc = smem_desc_kmajor_sw128(tiles_b + s * kTileB);
#pragma unroll
      for (int kk = 0; kk < kBK / 16; ++kk) {
        // +32 bytes per 16-element K step inside the swizzled row.
        umma_f16(tmem, a_desc + 2 * kk, b_desc + 2 * kk, idesc, (kb | kk) != 0);
      }
      umma_commit(&bars->empty[s]);
      *reinterpret_cast<volatile int*>(&bars->consumed) = kb + 1;
    }
    umma_commit(ok ? &bars->accum : &bars->drain);
    if (!ok) {
      volatile int never = 0;
      mbar_wait(&bars->drain, 0, &never, scratch, 4);
    }
  }
  __syncwarp();

  // Epilogue: all four warps, one TMEM lane quarter each.
  const bool ready = mbar_wait(&bars->accum, 0, abort, scratch, 5);
  __syncwarp();
  tc_fence_after_sync();
  if (ready) {
    const int row = m0 + warp * 32 + lane;
    const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;
#pragma unroll 1
    for (int c = 0; c < kBN; c += 32) {
      uint32_t v[32];
      tmem_load_32x32(tmem + lane_base + c, v);
      if (row < m) {
        __half* dst = out + static_cast<long long>(row) * n + n0 + c;
#pragma unroll
        for (int chunk = 0; chunk < 4; ++chunk) {
          if (n0 + c + chunk * 8 >= n) break;
          uint4 packed;
          __half2* h = reinterpret_cast<__half2*>(&packed);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            float a = __uint_as_float(v[chunk * 8 + 2 * j]);
            float b = __uint_as_float(v[chunk * 8 + 2 * j + 1]);
            if (kGelu) {
              a = ctb::gelu_erf(a);
              b = ctb::gelu_erf(b);
            }
            h[j] = __floats2half2_rn(a, b);
          }
          *reinterpret_cast<uint4*>(dst + chunk * 8) = packed;
        }
      }
    }
  }
  tc_fence_before_sync();
  __syncthreads();
  if (warp == 2) tmem_dealloc(tmem, kTmemCols);
}

}  // namespace

extern "C" __global__ void __launch_bounds__(kThreads, 1)
ctb_gemm_f16_tc(const __grid_constant__ TmaDescriptor tma_a, const __grid_constant__ TmaDescriptor tma_b,
                __half* output, int m, int n, int k, CTB_RESERVED_PARAMS) {
  (void)profile_scratch;
  gemm_tc<false>(&tma_a, &tma_b, output, m, n, k, runtime_scratch);
}

extern "C" __global__ void __launch_bounds__(kThreads, 1)
ctb_gemm_gelu_f16_tc(const __grid_constant__ TmaDescriptor tma_a, const __grid_constant__ TmaDescriptor tma_b,
                     __half* output, int m, int n, int k, CTB_RESERVED_PARAMS) {
  (void)profile_scratch;
  gemm_tc<true>(&tma_a, &tma_b, output, m, n, k, runtime_scratch);
}
