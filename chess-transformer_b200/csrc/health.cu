// The failure path of the library's bounded waits, on demand. Every kernel that waits on an mbarrier (a TMA load, an
// MMA commit, a cluster peer's arrival) gives up after the device's wait limit (g_wait_limit_ns, 2 s unless
// fry_set_wait_limit_ns changed it), records kWaitTimeout with the wait's site in the status word and returns, so a
// stalled kernel ends and the context stays usable. wait_probe_kernel takes that path deliberately: one thread waits on
// an mbarrier that expects one arrival nobody makes, so the wait always runs out, after about the limit.
#include "common.cuh"

namespace fry {

constexpr int kProbeSite = 90;  // the `where` the probe records

__global__ void wait_probe_kernel() {
    __shared__ __align__(8) uint64_t never;
    if (threadIdx.x != 0) return;
    mbar_init(&never, 1);
    fence_barrier_init();
    mbar_wait(&never, 0, kProbeSite);  // phase 0 completes on an arrival that never comes
}

cudaError_t wait_probe(cudaStream_t stream) {
    wait_probe_kernel<<<1, 32, 0, stream>>>();
    return cudaGetLastError();
}

}  // namespace fry
