// prefill_bf16.cu -- placeholder until the tcgen05 kernel lands.
#include "fo_common.cuh"
#include "fo_kernels.h"
extern "C" cudaError_t fo_launch_prefill_bf16(const float *, const uint16_t *, const uint16_t *, const float *, float *,
                                              int64_t, int64_t, int64_t, int64_t, int64_t, int, int, cudaStream_t) {
    return cudaErrorNotSupported;
}
