// FP16 GEMM / GEMM+GELU with FP32 accumulation on warp-level MMA (WMMA).
//
// Portable variant for any M, N, K: C[M,N] = A[M,K] . B[K,N] (row-major, no
// bias, transA = transB = 0), FP32 accumulator, optional exact-erf GELU on
// the accumulator, round-to-nearest FP16 store (python/cutriton/
// triton_kernels/transformer.py:17-107). The tcgen05 kernel (gemm_f16_tc.cu)
// is the fast path for tile-aligned shapes.

#include <mma.h>

#include "common.cuh"

namespace {

using namespace nvcuda;

constexpr int kBM = 128, kBN = 128, kBK = 32;
constexpr int kThreads = 256;  // 8 warps: 4 (M) x 2 (N), each 32 x 64

template <bool kGelu>
__device__ __forceinline__ void gemm_wmma(const __half* __restrict__ a, const __half* __restrict__ b,
                                          __half* __restrict__ c, int m, int n, int k) {
  __shared__ __align__(32) __half As[kBM][kBK + 8];
  __shared__ __align__(32) __half Bs[kBK][kBN + 8];
  __shared__ __align__(32) float Cs[8][32 * 64 / 8];  // per-warp staging, reused per fragment row
  const int warp = threadIdx.x / 32;
  const int wm = warp % 4, wn = warp / 4;
  const int m0 = blockIdx.x * kBM, n0 = blockIdx.y * kBN;
  const bool vec = ((k & 7) == 0) && ((n & 7) == 0) && ctb::aligned16(a) && ctb::aligned16(b);

  wmma::fragment<wmma::accumulator, 16, 16, 16, float> acc[2][4];
#pragma unroll
  for (int i = 0; i < 2; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) wmma::fill_fragment(acc[i][j], 0.0f);

  for (int k0 = 0; k0 < k; k0 += kBK) {
    // A tile: 128 x 32 halves = 512 vectors of 8.
    for (int e = threadIdx.x; e < kBM * kBK / 8; e += kThreads) {
      const int row = e / (kBK / 8), col = (e % (kBK / 8)) * 8;
      const int gm = m0 + row, gk = k0 + col;
      uint4 v = make_uint4(0, 0, 0, 0);
      if (vec) {
        if (gm < m && gk < k) v = *reinterpret_cast<const uint4*>(a + static_cast<long long>(gm) * k + gk);
      } else {
        __half* h = reinterpret_cast<__half*>(&v);
        for (int t = 0; t < 8; ++t) {
          if (gm < m && gk + t < k) h[t] = a[static_cast<long long>(gm) * k + gk + t];
        }
      }
      *reinterpret_cast<uint4*>(&As[row][col]) = v;
    }
    // B tile: 32 x 128 halves.
    for (int e = threadIdx.x; e < kBK * kBN / 8; e += kThreads) {
      const int row = e / (kBN / 8), col = (e % (kBN / 8)) * 8;
      const int gk = k0 + row, gn = n0 + col;
      uint4 v = make_uint4(0, 0, 0, 0);
      if (vec) {
        if (gk < k && gn < n) v = *reinterpret_cast<const uint4*>(b + static_cast<long long>(gk) * n + gn);
      } else {
        __half* h = reinterpret_cast<__half*>(&v);
        for (int t = 0; t < 8; ++t) {
          if (gk < k && gn + t < n) h[t] = b[static_cast<long long>(gk) * n + gn + t];
        }
      }
      *reinterpret_cast<uint4*>(&Bs[row][col]) = v;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < kBK; kk += 16) {
      wmma::fragment<wmma::matrix_a, 16, 16, 16, __half, wmma::row_major> fa[2];
      wmma::fragment<wmma::matrix_b, 16, 16, 16, __half, wmma::row_major> fb[4];
#pragma unroll
      for (int i = 0; i < 2; ++i) wmma::load_matrix_sync(fa[i], &As[wm * 32 + i * 16][kk], kBK + 8);
#pragma unroll
      for (int j = 0; j < 4; ++j) wmma::load_matrix_sync(fb[j], &Bs[kk][wn * 64 + j * 16], kBN + 8);
#pragma unroll
      for (int i = 0; i < 2; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) wmma::mma_sync(acc[i][j], fa[i], fb[j], acc[i][j]);
    }
    __syncthreads();
  }

  float* stage = Cs[warp];
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int i = 0; i < 2; ++i) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      wmma::store_matrix_sync(stage, acc[i][j], 16, wmma::mem_row_major);
      __syncwarp();
      for (int e = lane; e < 256; e += 32) {
        const int gm = m0 + wm * 32 + i * 16 + e / 16;
        const int gn = n0 + wn * 64 + j * 16 + e % 16;
        if (gm < m && gn < n) {
          const float v = stage[e];
          c[static_cast<long long>(gm) * n + gn] = __float2half_rn(kGelu ? ctb::gelu_erf(v) : v);
        }
      }
      __syncwarp();
    }
  }
}

}  // namespace

extern "C" __global__ void __launch_bounds__(kThreads)
ctb_gemm_f16_wmma(const __half* a, const __half* b, __half* output, int m, int n, int k, CTB_RESERVED_PARAMS) {
  CTB_UNUSED_RESERVED();
  CTB_GRID_DEPENDENCY_SYNC();
  gemm_wmma<false>(a, b, output, m, n, k);
}

extern "C" __global__ void __launch_bounds__(kThreads)
ctb_gemm_gelu_f16_wmma(const __half* a, const __half* b, __half* output, int m, int n, int k,
                       CTB_RESERVED_PARAMS) {
  CTB_UNUSED_RESERVED();
  CTB_GRID_DEPENDENCY_SYNC();
  gemm_wmma<true>(a, b, output, m, n, k);
}
