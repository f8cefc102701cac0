/*
 * dia_core.cuh -- shared machinery of the DIA kernels.
 *
 * Every product in this library (SpMV, diagonal-pair SpMSpM, the SIMT
 * dense-band product) is a "shifted-product sum" over output diagonals:
 *
 *     out[i] = sum_t  U[u_t + i] * V[v_t + i]      for rows i in [lo_t, hi_t)
 *
 * where a term t pairs a diagonal of A (aligned with the output row) with a
 * shifted diagonal of B or with the shifted x vector.  Any of the
 * reference's layouts (Recon, HM, row-packed) and the library's padded rows
 * layout reduces to a per-diagonal element offset plus a valid row range, so
 * one inner loop serves all of them.  The loop reads U and V with fully
 * coalesced loads (consecutive rows on consecutive lanes), keeps kILP rows
 * per thread in registers, and rounds every multiply and add separately in
 * term order, which reproduces the reference CPU loops bit for bit.
 */
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

namespace dia {

constexpr int kBlock = 256;          /* threads per CTA */
constexpr int kILP = 4;              /* rows per thread */
constexpr int kTile = kBlock * kILP; /* rows per tile */
constexpr int kBatch = 4;            /* terms whose loads are issued together */
constexpr int kMaxTerms = 384;       /* terms staged in shared memory at once */

/* One term of an output diagonal: element offsets of U and V at row 0 and
 * the rows where both operands exist. */
struct Term {
    long long u;
    long long v;
    int lo;
    int hi;
};

/* One output diagonal: element offset of row 0, rows that carry a value
 * [olo, ohi), rows written [wlo, whi) (zero where not valid: padding), and
 * its term range [t0, t1) in the term array. */
struct OutDesc {
    long long o;
    int olo, ohi;
    int wlo, whi;
    int t0, t1;
};

__device__ __forceinline__ float mul_add_rn(float acc, float a, float b)
{
    return __fadd_rn(acc, __fmul_rn(a, b));
}

/* Accumulate terms [0, nt) held in shared memory into acc for the rows
 * r0 + j*kBlock (j < kILP) of the tile [tile_lo, tile_lo + kTile).
 * Terms are taken kBatch at a time: when every term of a batch covers the
 * whole tile, all kBatch*kILP*2 loads are issued before the first multiply,
 * so one memory latency is paid per batch instead of per term; the adds are
 * still applied term by term in list order.  Terms that cover the tile only
 * partly take the per-row checked path; others are skipped. */
template <bool STREAM_U, int ILP = kILP, int BATCH = kBatch>
__device__ __forceinline__ void accumulate_terms(const float* __restrict__ U,
                                                 const float* __restrict__ V,
                                                 const Term* s_terms, int nt,
                                                 int tile_lo, int r0,
                                                 float (&acc)[ILP])
{
    constexpr int kTile = kBlock * ILP;
    constexpr int kILP = ILP;
    constexpr int kBatch = BATCH;
    const int tile_hi = tile_lo + kTile;
    int q = 0;
    for (; q + kBatch <= nt; q += kBatch) {
        Term t[kBatch];
        bool full = true;
#pragma unroll
        for (int u = 0; u < kBatch; ++u) {
            t[u] = s_terms[q + u];
            full &= (t[u].lo <= tile_lo) & (tile_hi <= t[u].hi);
        }
        if (!full) break;
        float a[kBatch][kILP], b[kBatch][kILP];
#pragma unroll
        for (int u = 0; u < kBatch; ++u) {
            const float* __restrict__ up = U + t[u].u + r0;
            const float* __restrict__ vp = V + t[u].v + r0;
#pragma unroll
            for (int j = 0; j < kILP; ++j) {
                a[u][j] = STREAM_U ? __ldcs(up + j * kBlock) : __ldg(up + j * kBlock);
                b[u][j] = __ldg(vp + j * kBlock);
            }
        }
#pragma unroll
        for (int u = 0; u < kBatch; ++u)
#pragma unroll
            for (int j = 0; j < kILP; ++j) acc[j] = mul_add_rn(acc[j], a[u][j], b[u][j]);
    }
    for (; q < nt; ++q) {
        const Term t = s_terms[q];
        if (t.lo <= tile_lo && tile_hi <= t.hi) {
            const float* __restrict__ up = U + t.u + r0;
            const float* __restrict__ vp = V + t.v + r0;
            float a[kILP], b[kILP];
#pragma unroll
            for (int j = 0; j < kILP; ++j) {
                a[j] = STREAM_U ? __ldcs(up + j * kBlock) : __ldg(up + j * kBlock);
                b[j] = __ldg(vp + j * kBlock);
            }
#pragma unroll
            for (int j = 0; j < kILP; ++j) acc[j] = mul_add_rn(acc[j], a[j], b[j]);
        } else if (t.lo < tile_hi && tile_lo < t.hi) {
#pragma unroll
            for (int j = 0; j < kILP; ++j) {
                const int i = r0 + j * kBlock;
                if (i >= t.lo && i < t.hi) {
                    const float a = STREAM_U ? __ldcs(U + t.u + i) : __ldg(U + t.u + i);
                    const float b = __ldg(V + t.v + i);
                    acc[j] = mul_add_rn(acc[j], a, b);
                }
            }
        }
    }
}

/* ---------------------------------------------------------------- host */

void set_error(const std::string& msg);
int fail(int code, const std::string& msg);
int cuda_fail(cudaError_t e, const char* what);
int num_sms();
int persistent_blocks(const void* kernel, int smem_bytes);

/* Persistent pair-sum kernel over nOut output diagonals and rows
 * [row_lo, row_hi) (spmspm.cu).  With nOut_dev the count is read on the
 * device and nOut is a capacity.  rows_per_thread is 4 or 8 (8 measured
 * faster on matrix-power chain steps, 1.84 -> 1.55 ms for H^8 of the
 * config-1 operator, and slower on the scattered config-3 product). */
int launch_pair_sum(const float* U, const float* V, float* O, const OutDesc* outs,
                    const Term* terms, int nOut, int row_lo, int row_hi, bool accumulate,
                    cudaStream_t stream, float avg_terms = -1.0f,
                    const int* nOut_dev = nullptr, int rows_per_thread = 4);

/* Term lists of a rows-layout product written into caller buffers (terms:
 * nC * nA slots, outs: nC), built on the device in A storage order
 * (spmspm.cu).  With nA_dev / nC_dev the counts are read on the device and
 * nA / nC are capacities. */
int build_generic_terms_rows(long long n, const int* d_A_off, int nA, const int* d_B_off, int nB,
                             const int* d_C_off, int nC, long long A_stride,
                             long long B_stride, long long b_vrow0, long long b_lo,
                             long long b_hi, long long C_stride, long long vrow0,
                             long long row_lo, long long row_hi, Term* terms, OutDesc* outs,
                             cudaStream_t stream, const int* nA_dev = nullptr,
                             const int* nC_dev = nullptr);

}  // namespace dia

#define DIA_TRY_CUDA(expr)                                   \
    do {                                                     \
        cudaError_t e__ = (expr);                            \
        if (e__ != cudaSuccess) return dia::cuda_fail(e__, #expr); \
    } while (0)
