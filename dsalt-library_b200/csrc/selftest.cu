// Self-test of the failure path of every tensor-core kernel: the bounded
// mbarrier wait (sm100::mbar_wait, the same function the kernels use).  One CTA
// initialises a barrier that nothing ever arrives on and waits on it; the wait
// gives up after its limit (about 2 s of SM clocks), sets DSALT_DEV_WAIT_TIMEOUT
// in the status word and returns, and the kernel exits normally, so the
// context stays usable.  No trap, no fault, no unbounded loop.
#include "common.cuh"
#include "sm100.cuh"

namespace dsalt {
namespace {

__global__ void __launch_bounds__(32) wait_timeout_probe_kernel(int32_t* status) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  const uint32_t b = sm100::smem_u32(&bar);
  if (threadIdx.x == 0) {
    sm100::mbar_init(b, 1);
    abort_flag = 0;
    sm100::fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    // phase 0 never completes: the bounded wait returns false after its limit
    (void)sm100::mbar_wait(b, 0, &abort_flag, status);
  }
  __syncthreads();
}

}  // namespace

cudaError_t launch_wait_timeout_probe(int32_t* status, cudaStream_t st) {
  wait_timeout_probe_kernel<<<1, 32, 0, st>>>(status);
  return cudaGetLastError();
}

}  // namespace dsalt
