// Self-test of the bounded-wait machinery: a wait that runs out must end the kernel with
// HMB_ERR_TIMEOUT in the device status word and leave the context usable. The kernel waits on an
// mbarrier that nothing arrives on (the "flag that nothing sets"), with the same try_wait loop and
// %globaltimer limit as the GEMM and GEMV rings, but a caller-chosen limit of at most 100 ms.
#include "common.cuh"

namespace hmb {
namespace {

__global__ void bounded_wait_kernel(int *status, uint64_t limit_ns) {
    __shared__ __align__(8) uint64_t bar;
    if (threadIdx.x != 0) return;
    const uint32_t b = static_cast<uint32_t>(__cvta_generic_to_shared(&bar));
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(b) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    uint64_t start;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(start));
    for (;;) {
        uint32_t done;
        asm volatile("{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], 0; selp.u32 %0, 1, 0, p; }"
                     : "=r"(done)
                     : "r"(b)
                     : "memory");
        if (done) return;  // cannot happen: no thread arrives
        uint64_t now;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(now));
        if (now - start > limit_ns) {
            atomicOr(status, 1);
            return;
        }
    }
}

}  // namespace
}  // namespace hmb

using namespace hmb;

extern "C" int hmb_selftest_bounded_wait(int64_t limit_ns, hmb_stream_t stream) {
    if (limit_ns <= 0 || limit_ns > 100000000) return HMB_ERR_ARG;
    int *status = device_status_word();
    if (!status) return HMB_ERR_CUDA;
    bounded_wait_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(status, static_cast<uint64_t>(limit_ns));
    return launch_status();
}
