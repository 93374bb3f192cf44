// tcgen05 tensor-core GEMM (placeholder until the kernel lands).
#include "common.cuh"
#include "ops.h"

namespace shield {

bool gemm_tc_supports(const DevWeight &w, int64_t M) { return false; }

cudaError_t launch_gemm_tc(const DevWeight &w, const QAct &q, float *y, int64_t ldy, int epi, int32_t *err,
                           cudaStream_t s) {
    return cudaErrorNotSupported;
}

cudaError_t launch_block_dots_tc(const DevWeight &w, const QAct &q, int32_t *dots, int32_t *err, cudaStream_t s) {
    return cudaErrorNotSupported;
}

}  // namespace shield
