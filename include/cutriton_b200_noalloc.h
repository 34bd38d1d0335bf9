/* No-allocation FP16 GEMM entry point (libcutriton_b200_noalloc.so).
 *
 * This call has no counterpart in the reference: it is an addition of this
 * backend for callers that must not allocate device or pinned memory on the
 * call path (a serving loop with a fixed memory footprint, a locked-down
 * allocator). It runs the same persistent tcgen05 FP16 GEMM as the engine's
 * "Gemm"/"GemmGelu" ops, with the kernel's scratch (its 64-byte error block)
 * in a 256-byte static device array instead of an engine-owned buffer.
 *
 *   C[m, n] = A[m, k] . B[k, n]  (optionally erf-GELU), FP16 in/out, FP32 accumulate
 *
 * a:   A, row-major [m, k] FP16, device pointer, 16-byte aligned
 * b_t: B transposed, row-major [n, k] FP16 (K-major), 16-byte aligned
 * c:   C, row-major [m, n] FP16, 16-byte aligned
 * k, n: multiples of 8. apply_gelu: 0 or 1. stream: a cudaStream_t (NULL = legacy)
 * of the current device; a stream of another device is rejected with
 * CTB_NOALLOC_INVALID_ARGUMENT.
 * error/error_len: optional caller buffer for a message when the result is nonzero.
 *
 * Synchronous on `stream`; returns CTB_NOALLOC_OK (0) on success. The first
 * call on a device does its set-up and should precede any stream capture;
 * calls overlapping in time on one device race on the shared scratch array and
 * must be serialised by the caller.
 */
#ifndef CUTRITON_B200_NOALLOC_H_
#define CUTRITON_B200_NOALLOC_H_

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

enum ctb_noalloc_code {
  CTB_NOALLOC_OK = 0,
  CTB_NOALLOC_INVALID_ARGUMENT = 1,
  CTB_NOALLOC_SCRATCH_TOO_SMALL = 2,
  CTB_NOALLOC_CUDA_ERROR = 3,
  CTB_NOALLOC_KERNEL_ERROR = 4,
};

int ctb_gemm_f16_noalloc(const void* a, const void* b_t, void* c, int m, int n, int k, int apply_gelu,
                         void* stream, char* error, size_t error_len);

#ifdef __cplusplus
}
#endif

#endif /* CUTRITON_B200_NOALLOC_H_ */
