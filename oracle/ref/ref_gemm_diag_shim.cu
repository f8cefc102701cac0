/*
 * ref_gemm_diag_shim.cu -- TEST INFRASTRUCTURE: exposes gemm_diag's host
 * routines and kernel through a C ABI (compiled from the reference sources
 * where they lie; output in oracle/_ref/, not committed).
 *
 *   gemm_diag/gemm_diag.cu:334-356  cpu_diag_multiply (dense n x n)
 *   gemm_diag/gemm_diag.cu:361-382  pack_diag_matrix (mt19937, U(0.5,1.5))
 *   gemm_diag/gemm_diag.cu:387-423  build_c_layout
 *   gemm_diag/gemm_diag.cu:119-329  gemm_diag_kernel
 */
#include <cstring>
#include <vector>
#define main ref_main_gemm_diag
#include "gemm_diag/gemm_diag.cu"
#undef main

extern "C" {

void ref_pack_diag_matrix(int n, int P, const int* offsets, unsigned seed,
                          float* DA)
{
    std::vector<int> off(offsets, offsets + P), off_out;
    std::vector<float> out;
    pack_diag_matrix(n, off, seed, out, off_out);
    std::memcpy(DA, out.data(), out.size() * sizeof(float));
}

int ref_build_c_layout(int n, int P, const int* off_A, int Q, const int* off_B,
                       int* C_offsets, int* C_lens, int* k_to_idx, int* k_list,
                       int* total_c)
{
    std::vector<int> a(off_A, off_A + P), b(off_B, off_B + Q), co, cl, k2i, kl;
    int tot = 0, num_k = 0;
    build_c_layout(n, a, b, co, cl, k2i, tot, num_k, kl);
    for (int i = 0; i < num_k; ++i) {
        if (C_offsets) C_offsets[i] = co[i];
        if (C_lens) C_lens[i] = cl[i];
        if (k_list) k_list[i] = kl[i];
    }
    if (k_to_idx) std::memcpy(k_to_idx, k2i.data(), k2i.size() * sizeof(int));
    if (total_c) *total_c = tot;
    return num_k;
}

/* Dense n x n result of cpu_diag_multiply (n <= 4096 as in the reference). */
void ref_cpu_diag_multiply(const float* DA, const int* off_A, int P,
                           const float* DB, const int* off_B, int Q, int n,
                           float* C_dense)
{
    std::vector<float> out;
    cpu_diag_multiply(DA, off_A, P, DB, off_B, Q, n, out);
    std::memcpy(C_dense, out.data(), out.size() * sizeof(float));
}

/* The reference kernel, launched exactly as its main does (C zeroed by the
 * caller; the kernel accumulates with atomics). */
int ref_launch_gemm_diag(const float* DA, const float* DB, const int* offA,
                         const int* offB, int P, int Q, int n, float* C,
                         const int* C_off, const int* C_len, const int* k2idx,
                         void* stream)
{
    int num_a_tiles = (P + TI - 1) / TI;
    int num_col_tiles = (n + TC - 1) / TC;
    dim3 grid(num_a_tiles, num_col_tiles);
    gemm_diag_kernel<<<grid, BLOCK_SIZE, 0, (cudaStream_t)stream>>>(
        DA, DB, offA, offB, P, Q, n, C, C_off, C_len, k2idx, num_a_tiles,
        num_col_tiles);
    return (int)cudaGetLastError();
}

}  // extern "C"
