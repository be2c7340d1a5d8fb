// Self-test of the library's failure path: a wait that nothing satisfies gives up, records a status and returns.
//
// One CTA of two warps.  Each warp's first lane waits, through the same bounded mbar_wait every kernel of the
// library uses, on an mbarrier of its own that no thread arrives on.  The first wait to pass the wait limit records
// CQ_ERR_TIMEOUT with its site (kSelftestSite + warp) in the device status word and raises the CTA's abort flag;
// the other wait sees the flag and returns without recording.  No global memory besides the status word is touched,
// so the context stays usable and the caller reads the failure with cq_take_device_status().
#include "kernels.cuh"

namespace cq {

__global__ void __launch_bounds__(64) selftest_wait_kernel() {
  __shared__ uint64_t bars[2];
  __shared__ int abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();
  if (lane == 0) mbar_wait(&bars[warp], 0u, &abort_flag, kSelftestSite + warp);
  __syncthreads();
}

cudaError_t launch_selftest_wait(cudaStream_t st) {
  selftest_wait_kernel<<<1, 64, 0, st>>>();
  return cudaGetLastError();
}

}  // namespace cq
