// sm_100a building blocks for the tensor-core kernels: mbarriers with
// bounded waits, TMA tile loads, and the 5th-generation tensor core
// (tcgen05: TMEM allocation, UMMA issue/commit, TMEM loads).
//
// Descriptor encodings follow the PTX ISA "tcgen05" matrix and instruction
// descriptor formats (also documented in CUTLASS cute/arch/mma_sm100_desc.hpp):
//   shared-memory descriptor: start>>4 [0,14), LBO>>4 [16,30), SBO>>4 [32,46),
//     version 1 [46,48), base offset [49,52), layout [61,64) (2 = 128B swizzle);
//   instruction descriptor (kind::f16 / kind::tf32): D format [4,6) (1 = F32),
//     A format [7,10), B format [10,13) (0 = F16, 1 = BF16, 2 = TF32),
//     A major bit 15, B major bit 16 (0 = K-major), N>>3 [17,23), M>>4 [24,29).
//
// Every wait is bounded: after kWaitLimitNs of global time the waiting thread
// records kErrorWaitTimeout in the error block and reports failure, and the
// kernel unwinds (drains what it issued, frees TMEM, returns) instead of
// hanging. Every tensor copy fills the shared memory of the CTA that issues it.
#pragma once

#include "common.cuh"

namespace ctb {
namespace tc {

constexpr unsigned long long kWaitLimitNs = 2000000000ull;  // 2 s

// CUtensorMap-compatible parameter (128 bytes, 64-byte aligned), passed as a
// __grid_constant__ kernel parameter and encoded by the host binder.
struct alignas(64) TmaDescriptor {
  unsigned long long opaque[16];
};

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long global_time_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---- mbarrier ---------------------------------------------------------------

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

// Makes barrier initialisation visible to the async proxy (TMA, tcgen05).
__device__ __forceinline__ void mbar_init_fence() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

// Waits for phase `parity` of `bar` to complete. Returns false (after
// recording the error) when the wait exceeds `limit_ns` or `abort` is set by
// another thread of the CTA.
__device__ __forceinline__ bool mbar_wait_for(uint64_t* bar, uint32_t parity, volatile int* abort, void* scratch,
                                              unsigned int site, unsigned long long limit_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long start = global_time_ns();
  for (uint32_t spin = 1;; ++spin) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((spin & 255u) == 0) {
      if (*abort) return false;
      if (global_time_ns() - start > limit_ns) {
        *abort = 1;
        report_error(scratch, kErrorWaitTimeout, site);
        return false;
      }
    }
  }
}

__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort, void* scratch,
                                          unsigned int site) {
  return mbar_wait_for(bar, parity, abort, scratch, site, kWaitLimitNs);
}

// ---- TMA ----------------------------------------------------------------------

__device__ __forceinline__ void tma_prefetch(const TmaDescriptor* desc) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(desc)) : "memory");
}

__device__ __forceinline__ void tma_load_2d(void* dst, const TmaDescriptor* desc, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];"
      ::"r"(smem_addr(dst)), "l"(reinterpret_cast<uint64_t>(desc)), "r"(smem_addr(bar)), "r"(x), "r"(y)
      : "memory");
}

__device__ __forceinline__ void tma_load_3d(void* dst, const TmaDescriptor* desc, uint64_t* bar, int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];"
      ::"r"(smem_addr(dst)), "l"(reinterpret_cast<uint64_t>(desc)), "r"(smem_addr(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}

__device__ __forceinline__ void tma_load_4d(void* dst, const TmaDescriptor* desc, uint64_t* bar, int x, int y, int z,
                                            int w) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, %6}], "
      "[%2];" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(desc)), "r"(smem_addr(bar)), "r"(x), "r"(y), "r"(z), "r"(w)
      : "memory");
}

// ---- tcgen05 ------------------------------------------------------------------

// Whole-warp TMEM allocation; the base address is written to *dst (smem).
__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t columns) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(dst)),
               "r"(columns)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t columns) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(columns) : "memory");
}

__device__ __forceinline__ void tc_fence_before_sync() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after_sync() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem] . B[smem]^T, FP16/BF16 inputs (kind::f16).
__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D[tmem] (+)= A[smem] . B[smem]^T, TF32 inputs (kind::tf32).
__device__ __forceinline__ void umma_tf32(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrives once on `bar` when every tcgen05.mma issued so far by this thread
// has completed (and its smem operands may be overwritten).
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
               : "memory");
}

// K-major operand tile in the 128-byte swizzle canonical layout: rows of
// 128 B, 8-row (1024 B) swizzle atoms stacked along M/N (SBO = 1024 B).
__device__ __forceinline__ uint64_t smem_desc_kmajor_sw128(const void* tile) {
  const uint64_t start = (smem_addr(tile) >> 4) & 0x3FFFu;
  const uint64_t lbo = 1;            // unused for swizzled K-major layouts
  const uint64_t sbo = 1024 >> 4;
  return start | (lbo << 16) | (sbo << 32) | (1ull << 46) | (2ull << 61);
}

// Instruction descriptor: FP32 accumulator, A/B format `ab_format`, both
// operands K-major, tile M x N.
__host__ __device__ constexpr uint32_t instr_desc(uint32_t ab_format, uint32_t m, uint32_t n) {
  return (1u << 4) | (ab_format << 7) | (ab_format << 10) | ((n >> 3) << 17) | ((m >> 4) << 24);
}

constexpr uint32_t kFormatF16 = 0;
constexpr uint32_t kFormatTF32 = 2;

// 32 lanes x 32 consecutive 32-bit columns: thread t of the warp receives
// row (lane base + t), columns [col, col + 32).
__device__ __forceinline__ void tmem_load_32x32(uint32_t taddr, uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
        "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]),
        "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]),
        "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

}  // namespace tc
}  // namespace ctb
