// Self-test of the device timeout path: the bounded mbarrier wait every warp-specialised kernel uses, on a phase
// that completes only if the caller asks for the arrival.  When the limit runs out the wait returns false and the
// kernel ORs SELFTEST_TIMEOUT into the status word, as the production kernels do with their own bits, and returns:
// nothing traps, nothing spins without a limit, and the context stays usable.
#include "kernels.h"
#include "tc.cuh"

namespace spq {

__global__ void k_wait_selftest(int arrive, unsigned long long limit_ns, int* status) {
    __shared__ uint64_t bar;
    if (threadIdx.x == 0) {
        tc::mbar_init(&bar, 1);
        tc::mbar_fence_init();
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        if (arrive) tc::mbar_arrive(&bar);
        if (!tc::mbar_wait(&bar, 0u, limit_ns)) atomicOr(status, SELFTEST_TIMEOUT);
    }
}

cudaError_t launch_wait_selftest(int arrive, unsigned long long limit_ns, int* status, cudaStream_t st) {
    k_wait_selftest<<<1, 32, 0, st>>>(arrive, limit_ns, status);
    return cudaGetLastError();
}

}  // namespace spq
