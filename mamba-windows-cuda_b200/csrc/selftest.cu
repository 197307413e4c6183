// Self-test of the bounded device waits: one CTA waits for an mbarrier phase that can
// never complete (the barrier expects one arrival and nothing arrives). The wait gives up
// after a short iteration limit, records ERR_WAIT_TMA in the error word and the kernel
// returns normally, so the host reads the status and the context stays usable. No GPU
// fault, trap or unbounded loop is involved.
#include "mwc_internal.h"
#include "mwc_tma.cuh"

namespace mwc {

constexpr unsigned SELFTEST_SPINS = 1u << 12;

__global__ void wait_selftest_kernel(int* err) {
    __shared__ __align__(8) uint64_t bar;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        fence_mbar_init();
    }
    __syncthreads();
    if (threadIdx.x == 0) mbar_wait(&bar, 0u, err, SELFTEST_SPINS);
}

cudaError_t launch_wait_selftest(int* err, cudaStream_t s) {
    wait_selftest_kernel<<<1, 32, 0, s>>>(err);
    return cudaGetLastError();
}

}  // namespace mwc
