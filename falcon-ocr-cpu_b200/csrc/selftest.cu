// selftest.cu -- the bounded-wait self-test: one CTA waits on an mbarrier
// that nothing ever completes, gives up after the caller's limit, raises the
// context's error word and returns.  It proves on the device that a wait
// which runs out ends with an error status the host reads, and that the
// context stays usable afterwards (no trap, no fault, no hang).
#include "fo_kernels.h"
#include "sm100.cuh"

namespace fo {

__global__ void bounded_wait_kernel(unsigned *err, unsigned long long limit_ns) {
    __shared__ uint64_t bar;
    __shared__ int abort_flag;
    if (threadIdx.x == 0) {
        sm100::mbar_init(&bar, 1);  // one arrival expected; none ever comes
        abort_flag = 0;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        const bool ok = sm100::mbar_wait(&bar, 0, &abort_flag, err, limit_ns);
        if (!ok) {
            // Complete the phase ourselves so the barrier is left consistent.
            sm100::mbar_arrive(&bar);
        }
    }
    __syncthreads();
}

}  // namespace fo

extern "C" cudaError_t fo_launch_bounded_wait(unsigned *err, unsigned long long limit_ns, cudaStream_t stream) {
    fo::bounded_wait_kernel<<<1, 32, 0, stream>>>(err, limit_ns);
    return cudaGetLastError();
}
