// k_selftest.cu -- the failure-path self-test behind q3cu_selftest_wait_timeout.
//
// Every wait in the library's kernels is mbar_wait: bounded by a time limit
// (and a poll count), after which it sets Q3CU_DEV_TIMEOUT in the context's
// status word and returns false, and the kernel winds down.  This kernel makes
// that path run on purpose: its threads wait on an initialised barrier that no
// thread ever arrives on, so every wait gives up at the limit.  Nothing is
// out of bounds, nothing traps; the context is usable afterwards.
#include "q3cu_internal.h"

namespace q3 {

__global__ void selftest_wait_kernel(uint32_t *status) {
    __shared__ __align__(8) uint64_t never;
    if (threadIdx.x == 0) {
        mbar_init(&never, 1);
        mbar_init_fence();
    }
    __syncthreads();
    mbar_wait(&never, 0, threadIdx.x == 0 ? status : nullptr);   // gives up after the limit
}

cudaError_t launch_selftest_wait(uint32_t *status, cudaStream_t stream) {
    selftest_wait_kernel<<<1, 32, 0, stream>>>(status);
    return cudaGetLastError();
}

}  // namespace q3
