// selftest.cu -- exercises the failure path of the bounded waits without faulting the GPU:
// one thread waits on an mbarrier that nothing ever arrives at, with a short limit; the wait
// gives up, records its code in the device status word and the kernel returns normally.
#include "host_common.h"
#include "sm100.cuh"

namespace morpho {
namespace {

__global__ void wait_timeout_kernel(uint32_t* status, uint64_t limit_ns) {
    __shared__ __align__(8) uint64_t bar;
    if (threadIdx.x == 0) {
        const uint32_t b = smem_u32(&bar);
        mbar_init(b, 1);
        fence_barrier_init();
        // phase 0 never completes: nobody arrives
        mbar_wait_for(b, 0, limit_ns, status, K_SELFTEST, 1);
    }
}

}  // namespace
}  // namespace morpho

extern "C" int morpho_sm100_selftest_wait_timeout(uint32_t limit_us, void* stream) {
    using namespace morpho;
    clear_error();
    if (limit_us == 0 || limit_us > 1000000u)
        return set_error(MORPHO_ERR_INVALID, "limit_us must be in (0, 1000000]");
    DeviceInfo dev;
    MORPHO_TRY(current_device_info(&dev));
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    wait_timeout_kernel<<<1, 32, 0, st>>>(dev.status, static_cast<uint64_t>(limit_us) * 1000ull);
    MORPHO_CUDA_TRY(cudaGetLastError());
    return MORPHO_OK;
}
