// Self-test of the bounded device waits (the failure-detection path of every
// kernel here): one CTA waits on an mbarrier that nothing arrives on, with a
// caller-chosen limit.  The wait gives up, records kDevErrTimeout in the
// status word and the kernel returns normally, so the context stays usable
// and the host learns of the timeout through moe_check_device_status, as it
// would after a real stalled pipeline.  No fault, trap or unbounded spin.
#include "moe_internal.h"
#include "sm100.cuh"

namespace moe {
namespace {

using namespace sm100;

__global__ void __launch_bounds__(64) wait_selftest_kernel(int* status, uint64_t timeout_ns) {
    __shared__ __align__(8) uint64_t bar;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        fence_mbar_init();
    }
    __syncthreads();
    // warp 0: the stalled consumer; warp 1 does nothing (the producer that never arrives)
    if (threadIdx.x < 32) (void)__all_sync(0xffffffffu, mbar_wait_for(&bar, 0, status, kDevErrTimeout, timeout_ns));
}

}  // namespace

cudaError_t launch_wait_selftest(int* status, uint64_t timeout_ns, cudaStream_t st) {
    wait_selftest_kernel<<<1, 64, 0, st>>>(status, timeout_ns);
    return cudaGetLastError();
}

}  // namespace moe
