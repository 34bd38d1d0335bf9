// Failure-detection probe (op "BoundedWaitProbe"): the host-visible path a
// pipeline kernel takes when one of its waits can never be satisfied.
//
// Block 0 waits on a shared-memory mbarrier that nothing arrives on, with the
// same bounded-wait routine the tensor-core kernels use but a limit of
// `limit_us` microseconds; when it expires the routine records
// kErrorWaitTimeout (site 90) in the engine's error block and returns. The
// kernel then completes normally (every block copies its slice of x to the
// output), so no fault, trap or hang is involved: the host reads the error
// block at Synchronize and the context stays usable.

#include "tc_common.cuh"

extern "C" __global__ void __launch_bounds__(256)
ctb_bounded_wait_probe_f32(const float* x, float* output, int numel, int limit_us, CTB_RESERVED_PARAMS) {
  (void)profile_scratch;
  CTB_GRID_DEPENDENCY_SYNC();
  using namespace ctb::tc;
  __shared__ uint64_t never_completed;
  __shared__ int abort;
  if (threadIdx.x == 0) {
    mbar_init(&never_completed, 1);
    abort = 0;
    mbar_init_fence();
  }
  __syncthreads();
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    const unsigned long long limit_ns = static_cast<unsigned long long>(limit_us > 0 ? limit_us : 1) * 1000ull;
    mbar_wait_for(&never_completed, 0, &abort, runtime_scratch, 90, limit_ns);
  }
  __syncthreads();
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < numel;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    output[i] = x[i];
  }
}
