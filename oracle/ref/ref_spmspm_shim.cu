/*
 * ref_spmspm_shim.cu -- TEST INFRASTRUCTURE: exposes the reference's
 * SpMSpM host routines and GPU kernels through a C ABI (compiled from the
 * reference sources where they lie; output in oracle/_ref/, not committed).
 *
 *   spmspm/bench_spmspm.cu:89-131   make_banded, make_c_structure
 *   spmspm/bench_spmspm.cu:376-408  cpu_dia_spgemm (the OpenMP CPU oracle)
 *   spmspm/bench_spmspm.cu:349-368  dense_ref_to_cdiag
 *   spmspm/paper_hm.cuh:87-130      compute_c_hm_structure
 *   spmspm/spmspm.cu:256-319        gather_meta_kernel<512>
 *   spmspm/paper_hm_kernel.cu:31-93 hm_structured_sparse_matmul_kernel
 */
#include <cstring>
#include <vector>
#define main ref_main_bench_spmspm
#include "spmspm/bench_spmspm.cu"
#undef main

namespace {
DiaMatrix to_dia(int n, int K, const int* off, const int* len,
                 const long long* start, const float* val)
{
    DiaMatrix M;
    M.n = n;
    M.offsets.assign(off, off + K);
    M.lengths.assign(len, len + K);
    M.starts.resize(K);
    size_t nnz = 0;
    for (int k = 0; k < K; ++k) {
        M.starts[k] = (size_t)start[k];
        nnz = std::max(nnz, (size_t)start[k] + (size_t)len[k]);
    }
    M.values.assign(val, val + nnz);
    M.nnz = nnz;
    return M;
}
}  // namespace

extern "C" {

/* make_banded(n, w, seed): offsets -w..w, std::mt19937 U(-1,1) values. */
long long ref_make_banded(int n, int w, unsigned seed, int* off, int* len,
                          long long* start, float* val)
{
    DiaMatrix M = make_banded(n, w, seed);
    for (size_t k = 0; k < M.offsets.size(); ++k) {
        off[k] = M.offsets[k]; len[k] = M.lengths[k];
        start[k] = (long long)M.starts[k];
    }
    if (val) std::memcpy(val, M.values.data(), M.values.size() * sizeof(float));
    return (long long)M.nnz;
}

/* make_c_structure: returns the number of C diagonals. */
int ref_make_c_structure(int n, int nA, const int* A_off, int nB,
                         const int* B_off, int* C_off, int* C_len,
                         long long* C_start)
{
    DiaMatrix A, B;
    A.n = B.n = n;
    A.offsets.assign(A_off, A_off + nA);
    B.offsets.assign(B_off, B_off + nB);
    DiaMatrix C = make_c_structure(A, B);
    for (size_t k = 0; k < C.offsets.size(); ++k) {
        if (C_off) C_off[k] = C.offsets[k];
        if (C_len) C_len[k] = C.lengths[k];
        if (C_start) C_start[k] = (long long)C.starts[k];
    }
    return (int)C.offsets.size();
}

/* compute_c_hm_structure (the Haque baseline's symbolic phase). */
int ref_compute_c_hm_structure(int n, int nA, const int* A_off, int nB,
                               const int* B_off, int* C_off, int* C_len,
                               int* C_start)
{
    HMMatrix A, B;
    A.n = B.n = n;
    A.num_diags = nA; B.num_diags = nB;
    A.diag_offsets.assign(A_off, A_off + nA);
    B.diag_offsets.assign(B_off, B_off + nB);
    HMMatrix C = compute_c_hm_structure(A, B, n);
    for (int k = 0; k < C.num_diags; ++k) {
        if (C_off) C_off[k] = C.diag_offsets[k];
        if (C_len) C_len[k] = C.diag_lengths[k];
        if (C_start) C_start[k] = C.diag_starts[k];
    }
    return C.num_diags;
}

/* cpu_dia_spgemm over HM arrays; C structure from make_c_structure. */
void ref_cpu_dia_spgemm(int n, int nA, const int* A_off, const int* A_len,
                        const long long* A_start, const float* A_val, int nB,
                        const int* B_off, const int* B_len,
                        const long long* B_start, const float* B_val, int nC,
                        const int* C_off, const int* C_len,
                        const long long* C_start, float* C_val)
{
    DiaMatrix A = to_dia(n, nA, A_off, A_len, A_start, A_val);
    DiaMatrix B = to_dia(n, nB, B_off, B_len, B_start, B_val);
    DiaMatrix C;
    C.n = n;
    C.offsets.assign(C_off, C_off + nC);
    C.lengths.assign(C_len, C_len + nC);
    C.starts.resize(nC);
    size_t nnz = 0;
    for (int k = 0; k < nC; ++k) {
        C.starts[k] = (size_t)C_start[k];
        nnz = std::max(nnz, (size_t)C_start[k] + (size_t)C_len[k]);
    }
    C.nnz = nnz;
    std::vector<float> out = cpu_dia_spgemm(A, B, C);
    std::memcpy(C_val, out.data(), out.size() * sizeof(float));
}

/* dense O(n^3) reference mapped to C's diagonal layout (n <= ~1024). */
void ref_dense_ref_to_cdiag(int n, int nA, const int* A_off, const int* A_len,
                            const long long* A_start, const float* A_val,
                            int nB, const int* B_off, const int* B_len,
                            const long long* B_start, const float* B_val,
                            int nC, const int* C_off, const int* C_len,
                            const long long* C_start, float* C_val)
{
    DiaMatrix A = to_dia(n, nA, A_off, A_len, A_start, A_val);
    DiaMatrix B = to_dia(n, nB, B_off, B_len, B_start, B_val);
    DiaMatrix C;
    C.n = n;
    C.offsets.assign(C_off, C_off + nC);
    C.lengths.assign(C_len, C_len + nC);
    C.starts.resize(nC);
    size_t nnz = 0;
    for (int k = 0; k < nC; ++k) {
        C.starts[k] = (size_t)C_start[k];
        nnz = std::max(nnz, (size_t)C_start[k] + (size_t)C_len[k]);
    }
    C.values.assign(nnz, 0.0f);
    C.nnz = nnz;
    std::vector<float> out = dense_ref_to_cdiag(A, B, C);
    std::memcpy(C_val, out.data(), out.size() * sizeof(float));
}

/* The reference's gather_meta_kernel<512> on device HM buffers (signed
 * offsets, size_t starts, B_lookup of size 2n-1), launched as the bench
 * launches it (spmspm/bench_spmspm.cu:576-586). */
int ref_launch_gather_meta(const float* Av, const size_t* As, const int* Ao,
                           const int* Al, int nA, const float* Bv,
                           const size_t* Bs, const int* Bl, const int* Blk,
                           float* Cv, const size_t* Cs, const int* Co,
                           const int* Cl, int nC, int n, void* stream)
{
    if (nA > 512) return -1;
    dim3 mblk(256);
    dim3 mgrid((n + 256 * 4 - 1) / (256 * 4), nC);
    gather_meta_kernel<512><<<mgrid, mblk, 0, (cudaStream_t)stream>>>(
        Av, As, Ao, Al, nA, Bv, Bs, Bl, Blk, Cv, Cs, Co, Cl, nC, n);
    return (int)cudaGetLastError();
}

/* The Haque HM atomic baseline (int32 starts; C must be zeroed). */
int ref_launch_hm(const float* Av, const int* Ao, const int* As, const int* Al,
                  int nA, const float* Bv, const int* Bo, const int* Bs,
                  const int* Bl, int nB, float* Cv, const int* Co,
                  const int* Cs, const int* Cl, int nC, const int* Clk,
                  int nzA, int n, void* stream)
{
    hm_structured_sparse_matmul_kernel<<<(nzA + 255) / 256, 256, 0,
                                         (cudaStream_t)stream>>>(
        Av, Ao, As, Al, nA, Bv, Bo, Bs, Bl, nB, Cv, Co, Cs, Cl, nC, Clk, nzA, n);
    return (int)cudaGetLastError();
}

}  // extern "C"
