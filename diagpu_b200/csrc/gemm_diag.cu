/*
 * gemm_diag.cu -- the gemm_diag product C = A*B (row-packed inputs,
 * HM-packed output) for sm_100a.
 *
 * Reference: gemm_diag_kernel (gemm_diag/gemm_diag.cu:119-329) computes
 *     C[k][t] += sum_{i+j=k} DA[i][t] * DB[j][t+i]
 * over 4x4 diagonal tiles and scatters with global atomicAdd (C zeroed by
 * the caller first).  Here:
 *   - the host reads the P+Q offsets (or takes host copies), lists every
 *     output diagonal k with its (ri, rj) pairs in ri order -- the order
 *     cpu_diag_multiply (gemm_diag/gemm_diag.cu:334-356) adds them -- and a
 *     small device kernel turns that list into term descriptors using the
 *     caller's C layout (k_to_idx, C_offsets, C_lens);
 *   - SIMT mode reuses the persistent pair-sum kernel of spmspm.cu: one
 *     register accumulator per output value, one store (or one
 *     read-add-store for beta = 1), no atomics, deterministic;
 *   - TCGEN05 mode (contiguous dense bands) is the tensor-core kernel in
 *     gemm_diag_tc.cu.
 */
#include <algorithm>
#include <vector>

#include "../../include/diagpu_b200.h"
#include "dia_core.cuh"

namespace dia {

int gemm_diag_tc_supported(const int* h_off_A, int P, const int* h_off_B, int Q, int n);
int gemm_diag_tc_launch(const float* d_DA, const float* d_DB, const int* h_off_A, int P,
                        const int* h_off_B, int Q, int n, float* d_C_data,
                        const int* d_C_offsets, const int* d_C_lens, const int* d_k_to_idx,
                        int beta, cudaStream_t stream);

/* Host plan: nOut output diagonals (value k, term range) and the pair
 * (ri, rj) of every term. */
struct GemmPlanDev {
    const int* out_k;     /* [nOut] */
    const int* out_t;     /* [nOut + 1] */
    const int* pair_ri;   /* [np] */
    const int* pair_rj;   /* [np] */
    const int* off_A;     /* device offsets */
    const int* off_B;
    const int* k_to_idx;  /* [2n-1] */
    const int* C_offsets; /* value starts */
    const int* C_lens;
    int nOut, np, n;
    OutDesc* outs;
    Term* terms;
};

/* One thread per output diagonal, then one thread per term. */
__global__ void gemm_plan_kernel(GemmPlanDev g)
{
    const long long tid = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    const long long stride = (long long)gridDim.x * blockDim.x;
    for (long long j = tid; j < g.nOut; j += stride) {
        const int k = g.out_k[j];
        const int ki = g.k_to_idx[k + g.n - 1];
        OutDesc od;
        od.t0 = g.out_t[j];
        od.t1 = g.out_t[j + 1];
        if (ki < 0) { /* caller's layout has no such diagonal: skip, as :313-314 */
            od.o = 0;
            od.olo = od.ohi = od.wlo = od.whi = 0;
            od.t1 = od.t0;
        } else {
            const int m = min(k, 0);
            od.o = (long long)g.C_offsets[ki] + m;
            od.olo = od.wlo = -m;
            od.ohi = od.whi = g.C_lens[ki] - m;
        }
        g.outs[j] = od;
    }
    for (long long q = tid; q < g.np; q += stride) {
        const int ri = g.pair_ri[q], rj = g.pair_rj[q];
        const int i = g.off_A[ri], jo = g.off_B[rj];
        Term t;
        t.u = (long long)ri * g.n;                /* DA[ri][row] */
        t.v = (long long)rj * g.n + i;            /* DB[rj][row + i] */
        /* rows where A[row, row+i] and B[row+i, row+i+j] exist */
        const int lo = max(max(0, -i), max(-i, -i - jo));
        const int hi = min(min(g.n, g.n - i), min(g.n - i, g.n - i - jo));
        t.lo = lo;
        t.hi = max(hi, lo);
        g.terms[q] = t;
    }
}

static int gemm_diag_simt(const float* d_DA, const float* d_DB, const int* d_off_A,
                          const int* d_off_B, const std::vector<int>& hA,
                          const std::vector<int>& hB, int n, float* d_C, const int* d_C_offsets,
                          const int* d_C_lens, const int* d_k_to_idx, int beta,
                          cudaStream_t stream)
{
    const int P = (int)hA.size(), Q = (int)hB.size();
    struct Trip { long long k; int ri, rj; };
    std::vector<Trip> t;
    t.reserve((size_t)P * Q);
    for (int ri = 0; ri < P; ++ri)
        for (int rj = 0; rj < Q; ++rj) {
            const long long k = (long long)hA[ri] + hB[rj];
            if (k > -(long long)n && k < (long long)n) t.push_back({k, ri, rj});
        }
    std::stable_sort(t.begin(), t.end(), [](const Trip& a, const Trip& b) { return a.k < b.k; });
    std::vector<int> ints;  /* out_k | out_t | pair_ri | pair_rj */
    std::vector<int> out_k, out_t;
    for (size_t q = 0; q < t.size(); ++q)
        if (q == 0 || t[q].k != t[q - 1].k) {
            out_k.push_back((int)t[q].k);
            out_t.push_back((int)q);
        }
    out_t.push_back((int)t.size());
    const int nOut = (int)out_k.size(), np = (int)t.size();
    if (nOut == 0) return DIA_OK;
    ints.insert(ints.end(), out_k.begin(), out_k.end());
    ints.insert(ints.end(), out_t.begin(), out_t.end());
    for (auto& x : t) ints.push_back(x.ri);
    for (auto& x : t) ints.push_back(x.rj);

    const size_t term_bytes = (size_t)std::max(np, 1) * sizeof(Term);
    const size_t out_bytes = (size_t)nOut * sizeof(OutDesc);
    const size_t int_bytes = ints.size() * sizeof(int);
    void* ws = nullptr;
    DIA_TRY_CUDA(cudaMallocAsync(&ws, term_bytes + out_bytes + int_bytes, stream));
    GemmPlanDev g{};
    g.terms = (Term*)ws;
    g.outs = (OutDesc*)((char*)ws + term_bytes);
    int* di = (int*)((char*)ws + term_bytes + out_bytes);
    g.out_k = di;
    g.out_t = di + nOut;
    g.pair_ri = di + 2 * nOut + 1;
    g.pair_rj = di + 2 * nOut + 1 + np;
    g.off_A = d_off_A;
    g.off_B = d_off_B;
    g.k_to_idx = d_k_to_idx;
    g.C_offsets = d_C_offsets;
    g.C_lens = d_C_lens;
    g.nOut = nOut;
    g.np = np;
    g.n = n;
    int rc = DIA_OK;
    cudaError_t e = cudaMemcpyAsync(di, ints.data(), int_bytes, cudaMemcpyHostToDevice, stream);
    if (e != cudaSuccess) rc = cuda_fail(e, "gemm_diag plan upload");
    if (rc == DIA_OK) {
        const int grid = std::min(1024, (std::max(nOut, np) + kBlock - 1) / kBlock);
        gemm_plan_kernel<<<std::max(grid, 1), kBlock, 0, stream>>>(g);
        e = cudaGetLastError();
        if (e != cudaSuccess) rc = cuda_fail(e, "gemm_plan_kernel launch");
    }
    if (rc == DIA_OK)
        rc = launch_pair_sum(d_DA, d_DB, d_C, g.outs, g.terms, nOut, 0, n, beta != 0, stream,
                             (float)np / nOut);
    /* the host int buffer must outlive the copy: wait for it */
    cudaError_t es = cudaStreamSynchronize(stream);
    cudaError_t ef = cudaFreeAsync(ws, stream);
    if (rc == DIA_OK && es != cudaSuccess) rc = cuda_fail(es, "cudaStreamSynchronize");
    if (rc == DIA_OK && ef != cudaSuccess) rc = cuda_fail(ef, "cudaFreeAsync");
    return rc;
}

}  // namespace dia

using namespace dia;

extern "C" int dia_gemm_diag_ex(const float* d_DA, const float* d_DB, const int* d_off_A,
                                const int* d_off_B, const int* h_off_A, const int* h_off_B,
                                int P, int Q, int n, float* d_C_data, const int* d_C_offsets,
                                const int* d_C_lens, const int* d_k_to_idx, int beta, int mode,
                                cudaStream_t stream)
{
    if (P < 0 || Q < 0 || n < 0) return fail(DIA_ERR_INVALID, "dia_gemm_diag: negative size");
    if (beta != 0 && beta != 1) return fail(DIA_ERR_INVALID, "dia_gemm_diag: beta must be 0 or 1");
    if (mode < DIA_GEMM_AUTO || mode > DIA_GEMM_TCGEN05)
        return fail(DIA_ERR_INVALID, "dia_gemm_diag: unknown mode");
    if (n == 0 || P == 0 || Q == 0) return DIA_OK;
    if (!d_DA || !d_DB || !d_off_A || !d_off_B || !d_C_data || !d_C_offsets || !d_C_lens ||
        !d_k_to_idx)
        return fail(DIA_ERR_INVALID, "dia_gemm_diag: null pointer");
    if ((long long)n + kTile >= (1LL << 31))
        return fail(DIA_ERR_UNSUPPORTED, "dia_gemm_diag: n beyond int32 range");
    std::vector<int> hA(P), hB(Q);
    if (h_off_A && h_off_B) {
        std::copy(h_off_A, h_off_A + P, hA.begin());
        std::copy(h_off_B, h_off_B + Q, hB.begin());
    } else {
        DIA_TRY_CUDA(cudaMemcpyAsync(hA.data(), d_off_A, P * sizeof(int), cudaMemcpyDeviceToHost, stream));
        DIA_TRY_CUDA(cudaMemcpyAsync(hB.data(), d_off_B, Q * sizeof(int), cudaMemcpyDeviceToHost, stream));
        DIA_TRY_CUDA(cudaStreamSynchronize(stream));
    }
    const bool tc_ok = gemm_diag_tc_supported(hA.data(), P, hB.data(), Q, n) == DIA_OK;
    if (mode == DIA_GEMM_TCGEN05 && !tc_ok) return DIA_ERR_UNSUPPORTED; /* message set */
    if (mode == DIA_GEMM_TCGEN05 || (mode == DIA_GEMM_AUTO && tc_ok))
        return gemm_diag_tc_launch(d_DA, d_DB, hA.data(), P, hB.data(), Q, n, d_C_data,
                                   d_C_offsets, d_C_lens, d_k_to_idx, beta, stream);
    return gemm_diag_simt(d_DA, d_DB, d_off_A, d_off_B, hA, hB, n, d_C_data, d_C_offsets,
                          d_C_lens, d_k_to_idx, beta, stream);
}

extern "C" int dia_gemm_diag(const float* d_DA, const float* d_DB, const int* d_off_A,
                             const int* d_off_B, int P, int Q, int n, float* d_C_data,
                             const int* d_C_offsets, const int* d_C_lens, const int* d_k_to_idx,
                             cudaStream_t stream)
{
    return dia_gemm_diag_ex(d_DA, d_DB, d_off_A, d_off_B, nullptr, nullptr, P, Q, n, d_C_data,
                            d_C_offsets, d_C_lens, d_k_to_idx, 1, DIA_GEMM_AUTO, stream);
}
