// Tensor-core prefill GEMM (placeholder until the tcgen05 kernel lands).
#include "q35cu_internal.h"

namespace q35cu {

int launch_gemm_fp8(const q35cu_weight *w, const uint16_t *Xb, uint32_t m, float *Y, cudaStream_t st)
{
    (void)w; (void)Xb; (void)m; (void)Y; (void)st;
    return set_error(Q35CU_ERR_UNSUPPORTED, "gemm_fp8: tensor-core path not built yet");
}

}  // namespace q35cu
