// Self-test of the give-up path every pipeline kernel here shares: a bounded mbarrier wait that expires raises the
// wait-timeout status bit and returns, so the context stays usable. The kernel waits on an mbarrier that no thread
// ever arrives on, for a caller-chosen limit, then reports exactly as a pipeline kernel does when its copies do not
// land. No fault, trap or unbounded wait is involved.
#include "q3_common.cuh"
#include "q3_kernels.h"

namespace q3 {

__global__ void bounded_wait_selftest_kernel(uint32_t* status, unsigned long long limit_ns) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);   // one arrival expected, none ever made: phase 0 never completes
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0 && !mbar_wait_bounded(&bar, 0, limit_ns)) atomicOr(status, kStatusWaitTimeout);
}

cudaError_t launch_bounded_wait_selftest(uint32_t* status, unsigned long long limit_ns, cudaStream_t stream) {
  bounded_wait_selftest_kernel<<<1, 32, 0, stream>>>(status, limit_ns);
  return cudaGetLastError();
}

}  // namespace q3
