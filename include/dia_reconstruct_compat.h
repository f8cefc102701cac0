/*
 * dia_reconstruct_compat.h -- C++-linkage drop-in for the reference SpMV
 * launcher.
 *
 * Declares ReconView and launch_tc_spmv_regdirect with exactly the layout and
 * signature of spmv/src/dia_reconstruct.cuh:112-118 and :139-144, so a
 * program written against the reference header (e.g. spmv/test/
 * test_tc_spmv.cu, spmv/bench/bench_cusparse.cu) links against
 * libdiagpu_b200.so instead of tc_spmv_regdirect_kernel.cu.  The library's
 * implementation computes y = A*x in FP32 (dia_spmv_recon); the reference
 * kernel computed in TF32.  Like the reference launcher it returns nothing:
 * launch errors surface through cudaGetLastError(), argument errors through
 * dia_last_error().
 */
#ifndef DIA_RECONSTRUCT_COMPAT_H
#define DIA_RECONSTRUCT_COMPAT_H

#include <cuda_runtime.h>

struct ReconView {
    int rows;
    int cols;
    int num_diags;
    const int* diag_offsets; /* [num_diags], device memory */
    const float* values;     /* num_diags * cols, device memory */
};

void launch_tc_spmv_regdirect(ReconView R, const float* d_x, int x_size,
                              float* d_y, cudaStream_t stream = 0);

#endif
