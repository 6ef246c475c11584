// Self-test of the bounded waits every kernel of this library uses (common.cuh: mbar_wait): one thread waits on an
// mbarrier that nothing ever arrives on. The wait gives up after its cycle limit (~2 s), records kErrTimeoutSelftest in
// the caller's error word, raises the CTA's abort flag and returns, and the kernel ends normally, so the CUDA context
// stays usable. status[0] = 1 if the wait returned true (never expected), 2 if it gave up; status[1] = the abort flag.
#include "../../include/belt_b200.h"
#include "common.cuh"
#include "launch.h"

namespace belt {

__global__ void selftest_wait_kernel(int* err, int* status) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const bool ok = mbar_wait(&bar, 0, &abort_flag, err, kErrTimeoutSelftest);   // phase 0 never completes
    status[0] = ok ? 1 : 2;
    status[1] = abort_flag;
  }
}

cudaError_t launch_selftest_wait(int* err, int* status, cudaStream_t stream) {
  selftest_wait_kernel<<<1, 32, 0, stream>>>(err, status);
  return cudaGetLastError();
}

}  // namespace belt
