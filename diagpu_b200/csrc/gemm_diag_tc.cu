/*
 * gemm_diag_tc.cu -- tcgen05 TF32 dense-band kernel (placeholder until the
 * tensor-core path lands: reports DIA_ERR_UNSUPPORTED so AUTO mode takes the
 * exact SIMT path).
 */
#include "../../include/diagpu_b200.h"
#include "dia_core.cuh"

namespace dia {

int gemm_diag_tc_supported(const int*, int, const int*, int, int)
{
    return fail(DIA_ERR_UNSUPPORTED, "dia_gemm_diag: tcgen05 dense-band path not built");
}

int gemm_diag_tc_launch(const float*, const float*, const int*, int, const int*, int, int,
                        float*, const int*, const int*, const int*, int, cudaStream_t)
{
    return fail(DIA_ERR_UNSUPPORTED, "dia_gemm_diag: tcgen05 dense-band path not built");
}

}  // namespace dia
