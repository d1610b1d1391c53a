// Failure-detection probe (no counterpart in the reference): one CTA waits on an mbarrier that nothing
// arrives on, bounded by `limit_ns` of wall time -- the bounded wait every pipeline barrier of this
// library uses, with a short limit. The wait runs out, records EG2_DEV_TIMEOUT_PROBE in the device
// status word, and the kernel returns normally, leaving the context usable. Nothing faults, traps or
// hangs: this is how a stalled pipeline surfaces as EG2_ERR_TIMEOUT on the host.
#include "common.cuh"

namespace eg2 {

__global__ void wait_timeout_probe_kernel(unsigned long long limit_ns) {
    __shared__ uint64_t bar;
    __shared__ int abort_flag;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        abort_flag = 0;
        fence_mbarrier_init();
    }
    __syncthreads();
    if (threadIdx.x == 0) mbar_wait_limit(&bar, 0, EG2_DEV_TIMEOUT_PROBE, &abort_flag, limit_ns);
    __syncthreads();
}

int wait_timeout_probe(unsigned long long limit_ns, cudaStream_t s) {
    wait_timeout_probe_kernel<<<1, 32, 0, s>>>(limit_ns);
    return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

}  // namespace eg2
