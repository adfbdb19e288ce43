// Diagnostics for the bounded device waits. Every wait in the library's kernels gives up after a
// limit, raises a site code in the device error word and lets its CTA unwind; this probe runs that
// same wait (mbar_wait_or_abort) on an mbarrier that nothing ever arrives at, with a short limit,
// so that a test can check the path end to end without a fault: the wait runs out, the code is
// raised, the kernel returns and the context stays usable.

#include "common.cuh"
#include "launch.h"
#include "sm100.cuh"

namespace gdn {

__global__ void bounded_wait_probe_kernel(long long limit) {
    using namespace sm100;
    __shared__ uint64_t bar;
    __shared__ int abort;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);  // one arrival would complete phase 0; none comes
        abort = 0;
        fence_mbar_init();
    }
    __syncthreads();
    if (!mbar_wait_or_abort(&bar, 0, kSiteProbe, &abort, true, limit)) atomicExch(&abort, 1);
    __syncthreads();
}

int launch_bounded_wait_probe(int64_t limit_cycles, cudaStream_t s) {
    bounded_wait_probe_kernel<<<1, 32, 0, s>>>((long long)limit_cycles);
    return launch_status();
}

}  // namespace gdn
