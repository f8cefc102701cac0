/*
 * spmv.cu -- FP32 DIA SpMV for sm_100a.
 *
 * HBM-streaming design: each CTA owns a tile of kTile consecutive rows; the
 * term list (one term per diagonal) is built once per CTA in shared memory;
 * every warp then streams 32 consecutive values of each diagonal (one
 * coalesced 128-byte line, read with evict-first loads because values are
 * used once) and the matching shifted window of x (read through L1/L2, where
 * the K shifted windows of neighbouring rows overlap).  There is no tensor
 * core work: y = A*x moves 4*(nnz + 2n) bytes for 2*nnz flops, far below the
 * B200 ridge point, so HBM bandwidth is the bound.
 *
 * Reference behaviour (spmv/src/tc_spmv_regdirect_kernel.cu:62-147): y
 * overwritten, terms whose column leaves [0, cols) or [0, x_size) dropped.
 * The reference computed in TF32 on mma.sync; this computes in FP32 with the
 * CPU reference's summation order (spmv/test/test_tc_spmv.cu:64-79 for the
 * Recon layout, spmv/bench/bench_cusparse.cu:119-126 for ascending offsets).
 */
#include "../../include/dia_reconstruct_compat.h"
#include "../../include/diagpu_b200.h"
#include "dia_core.cuh"

namespace dia {

/* operator size below which chained products keep the values in L2 */
constexpr long long kL2KeepBytes = 48LL << 20;

struct SpmvArgs {
    const float* vals;
    const float* x;
    float* y;
    const int* off;
    int K;
    int row_lo, row_hi;   /* rows computed */
    int clo, chi;         /* columns that carry a term */
    long long u_row0;     /* element offset of (k = 0, row 0) in vals */
    long long u_kstride;  /* element stride between diagonals */
    int u_shift_by_d;     /* 1: value of row i at vals[.. + i + d] (Recon) */
    long long x_base;     /* x element of column c is x[c - x_base] */
    long long y_base;     /* y element of row i is y[i - y_base] */
    float scale;          /* EPI: y = scale * (A x) and sum += y */
    float* sum;
    int cache_vals;       /* 1: values read with normal caching (kept in L2 across launches) */
};

template <bool STREAM, bool EPI = false>
__global__ void __launch_bounds__(kBlock) spmv_kernel(SpmvArgs a)
{
    __shared__ Term s_t[kMaxTerms];
    const int tile_lo = a.row_lo + (int)blockIdx.x * kTile;
    const int r0 = tile_lo + (int)threadIdx.x;
    float acc[kILP];
#pragma unroll
    for (int j = 0; j < kILP; ++j) acc[j] = 0.0f;

    for (int k0 = 0; k0 < a.K; k0 += kMaxTerms) {
        const int nt = min(kMaxTerms, a.K - k0);
        if (k0) __syncthreads();
        for (int q = threadIdx.x; q < nt; q += kBlock) {
            const int k = k0 + q;
            const int d = a.off[k];
            Term t;
            t.u = a.u_row0 + (long long)k * a.u_kstride + (a.u_shift_by_d ? d : 0);
            t.v = (long long)d - a.x_base;
            /* rows i with column i + d in [clo, chi), clipped to the rows
             * computed so no load ever leaves the caller's buffers */
            long long lo = (long long)a.clo - d, hi = (long long)a.chi - d;
            lo = lo < a.row_lo ? a.row_lo : lo;
            hi = hi > a.row_hi ? a.row_hi : hi;
            if (hi < lo) hi = lo;
            t.lo = (int)lo;
            t.hi = (int)hi;
            s_t[q] = t;
        }
        __syncthreads();
        accumulate_terms<STREAM>(a.vals, a.x, s_t, nt, tile_lo, r0, acc);
    }
#pragma unroll
    for (int j = 0; j < kILP; ++j) {
        const int i = r0 + j * kBlock;
        if (i < a.row_hi) {
            if (EPI) {
                const float v = __fmul_rn(a.scale, acc[j]);
                a.y[i - a.y_base] = v;
                a.sum[i - a.y_base] = __fadd_rn(a.sum[i - a.y_base], v);
            } else {
                a.y[i - a.y_base] = acc[j];
            }
        }
    }
}

static int launch_spmv(const SpmvArgs& a, cudaStream_t stream)
{
    const long long rows = (long long)a.row_hi - a.row_lo;
    if (rows <= 0) return DIA_OK;
    const long long grid = (rows + kTile - 1) / kTile;
    if (a.sum && a.cache_vals)
        spmv_kernel<false, true><<<(unsigned)grid, kBlock, 0, stream>>>(a);
    else if (a.sum)
        spmv_kernel<true, true><<<(unsigned)grid, kBlock, 0, stream>>>(a);
    else
        spmv_kernel<true><<<(unsigned)grid, kBlock, 0, stream>>>(a);
    DIA_TRY_CUDA(cudaGetLastError());
    return DIA_OK;
}

}  // namespace dia

using namespace dia;

extern "C" int dia_spmv_recon(int rows, int cols, int num_diags, const int* d_diag_offsets,
                              const float* d_values, const float* d_x, int x_size, float* d_y,
                              cudaStream_t stream)
{
    if (rows < 0 || cols < 0 || num_diags < 0 || x_size < 0)
        return fail(DIA_ERR_INVALID, "dia_spmv_recon: negative size");
    if (rows == 0) return DIA_OK;
    if (!d_y || (num_diags > 0 && (!d_diag_offsets || !d_values || !d_x)))
        return fail(DIA_ERR_INVALID, "dia_spmv_recon: null pointer");
    if ((long long)rows + kTile >= (1LL << 31))
        return fail(DIA_ERR_UNSUPPORTED, "dia_spmv_recon: rows beyond int32 range");
    SpmvArgs a{};
    a.vals = d_values;
    a.x = d_x;
    a.y = d_y;
    a.off = d_diag_offsets;
    a.K = num_diags;
    a.row_lo = 0;
    a.row_hi = rows;
    a.clo = 0;
    a.chi = cols < x_size ? cols : x_size;
    a.u_row0 = 0;
    a.u_kstride = cols;
    a.u_shift_by_d = 1;
    a.x_base = 0;
    a.y_base = 0;
    return launch_spmv(a, stream);
}

extern "C" int dia_spmv_rows(int64_t n_rows, int64_t n_cols, int num_diags, const int* d_offsets,
                             const float* d_vals, int64_t stride, int64_t vrow0, int64_t row_lo,
                             int64_t row_hi, const float* d_x, int64_t x_lo, int64_t x_hi,
                             float* d_y, cudaStream_t stream)
{
    if (n_rows < 0 || n_cols < 0 || num_diags < 0 || stride < 0)
        return fail(DIA_ERR_INVALID, "dia_spmv_rows: negative size");
    if (row_lo < 0) row_lo = 0;
    if (row_hi > n_rows) row_hi = n_rows;
    if (row_hi <= row_lo) return DIA_OK;
    if (row_lo < vrow0 || row_hi > vrow0 + stride)
        return fail(DIA_ERR_INVALID, "dia_spmv_rows: rows outside the stored block");
    if (!d_y || (num_diags > 0 && (!d_offsets || !d_vals || !d_x)))
        return fail(DIA_ERR_INVALID, "dia_spmv_rows: null pointer");
    if (n_rows + kTile >= (1LL << 31) || n_cols >= (1LL << 31))
        return fail(DIA_ERR_UNSUPPORTED, "dia_spmv_rows: dimensions beyond int32 range");
    SpmvArgs a{};
    a.vals = d_vals;
    a.x = d_x;
    a.y = d_y;
    a.off = d_offsets;
    a.K = num_diags;
    a.row_lo = (int)row_lo;
    a.row_hi = (int)row_hi;
    a.clo = (int)(x_lo > 0 ? x_lo : 0);
    a.chi = (int)(x_hi < n_cols ? x_hi : n_cols);
    if (a.chi < a.clo) a.chi = a.clo;
    a.u_row0 = -vrow0;
    a.u_kstride = stride;
    a.u_shift_by_d = 0;
    a.x_base = x_lo;
    a.y_base = vrow0;
    return launch_spmv(a, stream);
}

/* C++-linkage drop-in for the reference launcher (same mangled signature as
 * spmv/src/dia_reconstruct.cuh:139-144). */
void launch_tc_spmv_regdirect(ReconView R, const float* d_x, int x_size, float* d_y,
                              cudaStream_t stream)
{
    dia_spmv_recon(R.rows, R.cols, R.num_diags, R.diag_offsets, R.values, d_x, x_size, d_y,
                   stream);
}

/* Truncated Taylor series of exp(tA) x on the rows layout (whole matrix):
 *     v_0 = x,  v_j = (t / j) * (A v_{j-1}),  y = v_0 + v_1 + ... + v_m,
 * one fused launch per term (SpMV, scale, running sum), so y stays in HBM
 * and each term costs 4*(nnz + 4n) bytes.  Rounding per element: the SpMV
 * sum in offset storage order, then fl(c_j * s) with c_j = fl(t / j), then
 * fl(y + v_j) -- the order of the CPU restatement in the oracle. */
extern "C" int dia_expm_taylor(int64_t n, int num_diags, const int* d_offsets, const float* d_vals,
                               int64_t stride, float t, int m, const float* d_x, float* d_y,
                               float* d_work, cudaStream_t stream)
{
    if (n < 0 || num_diags < 0 || m < 0 || stride < n)
        return fail(DIA_ERR_INVALID, "dia_expm_taylor: bad sizes (stride must be >= n)");
    if (n == 0) return DIA_OK;
    if (!d_x || !d_y || (m > 0 && (!d_work || (num_diags > 0 && (!d_offsets || !d_vals)))))
        return fail(DIA_ERR_INVALID, "dia_expm_taylor: null pointer");
    if (n + kTile >= (1LL << 31))
        return fail(DIA_ERR_UNSUPPORTED, "dia_expm_taylor: n beyond int32 range");
    DIA_TRY_CUDA(cudaMemcpyAsync(d_y, d_x, (size_t)n * 4, cudaMemcpyDeviceToDevice, stream));
    /* every term reads the whole matrix again: when the values fit in
     * about half of L2 they are read with normal caching, so terms after
     * the first find them there; larger matrices stream (evict-first) */
    const bool cache = (long long)num_diags * stride * 4 <= kL2KeepBytes;
    const float* v = d_x;
    for (int j = 1; j <= m; ++j) {
        float* vn = d_work + (size_t)(j & 1) * (size_t)n;
        SpmvArgs a{};
        a.vals = d_vals;
        a.x = v;
        a.y = vn;
        a.off = d_offsets;
        a.K = num_diags;
        a.row_lo = 0;
        a.row_hi = (int)n;
        a.clo = 0;
        a.chi = (int)n;
        a.u_row0 = 0;
        a.u_kstride = stride;
        a.u_shift_by_d = 0;
        a.x_base = 0;
        a.y_base = 0;
        a.scale = t / (float)j;
        a.sum = d_y;
        a.cache_vals = cache;
        const int rc = launch_spmv(a, stream);
        if (rc) return rc;
        v = vn;
    }
    return DIA_OK;
}

/* ------------------------------------------------------------ complex64 */

namespace dia {

/* complex fp32 multiply-add, rounding spelled out so the CPU oracle can
 * follow it: re += fl(fl(ar*br) - fl(ai*bi)), im += fl(fl(ar*bi) + fl(ai*br)) */
__device__ __forceinline__ void cmul_add(float2& acc, float2 a, float2 b)
{
    const float pr = __fsub_rn(__fmul_rn(a.x, b.x), __fmul_rn(a.y, b.y));
    const float pi = __fadd_rn(__fmul_rn(a.x, b.y), __fmul_rn(a.y, b.x));
    acc.x = __fadd_rn(acc.x, pr);
    acc.y = __fadd_rn(acc.y, pi);
}

struct SpmvC64Args {
    const float2* vals;   /* [K][stride] */
    const float2* x;
    float2* y;
    const int* off;
    int K, n_rows, n_cols;
    long long stride;
    /* EPI: y = (-i c) * (A x) and sum += y  (a term of exp(-i t A) x) */
    float c;
    float2* sum;
};

constexpr int kC64Ilp = 2;
constexpr int kC64Tile = kBlock * kC64Ilp;

/* One CTA per tile of rows; terms (one per diagonal) staged in shared
 * memory; lanes read consecutive rows of each diagonal (8-byte values,
 * 256-byte coalesced runs) and the matching shifted x window. */
template <bool EPI>
__global__ void __launch_bounds__(kBlock) spmv_c64_kernel(SpmvC64Args a)
{
    __shared__ Term s_t[kMaxTerms];
    const int tile_lo = (int)blockIdx.x * kC64Tile;
    const int r0 = tile_lo + (int)threadIdx.x;
    float2 acc[kC64Ilp];
#pragma unroll
    for (int j = 0; j < kC64Ilp; ++j) acc[j] = make_float2(0.0f, 0.0f);
    for (int k0 = 0; k0 < a.K; k0 += kMaxTerms) {
        const int nt = min(kMaxTerms, a.K - k0);
        if (k0) __syncthreads();
        for (int q = threadIdx.x; q < nt; q += kBlock) {
            const int k = k0 + q;
            const int d = a.off[k];
            Term t;
            t.u = (long long)k * a.stride;
            t.v = d;
            t.lo = max(0, -d);
            t.hi = min(a.n_rows, a.n_cols - d);
            if (t.hi < t.lo) t.hi = t.lo;
            s_t[q] = t;
        }
        __syncthreads();
        for (int q = 0; q < nt; ++q) {
            const Term t = s_t[q];
#pragma unroll
            for (int j = 0; j < kC64Ilp; ++j) {
                const int i = r0 + j * kBlock;
                if (i >= t.lo && i < t.hi)
                    cmul_add(acc[j], __ldcs(a.vals + t.u + i), __ldg(a.x + t.v + i));
            }
        }
    }
#pragma unroll
    for (int j = 0; j < kC64Ilp; ++j) {
        const int i = r0 + j * kBlock;
        if (i >= a.n_rows) continue;
        if (EPI) {
            /* (-i c) * (s.x + i s.y) = c s.y - i c s.x */
            const float2 v = make_float2(__fmul_rn(a.c, acc[j].y), -__fmul_rn(a.c, acc[j].x));
            a.y[i] = v;
            float2 s = a.sum[i];
            s.x = __fadd_rn(s.x, v.x);
            s.y = __fadd_rn(s.y, v.y);
            a.sum[i] = s;
        } else {
            a.y[i] = acc[j];
        }
    }
}

static int launch_spmv_c64(const SpmvC64Args& a, cudaStream_t stream)
{
    if (a.n_rows <= 0) return DIA_OK;
    const long long grid = ((long long)a.n_rows + kC64Tile - 1) / kC64Tile;
    if (a.sum)
        spmv_c64_kernel<true><<<(unsigned)grid, kBlock, 0, stream>>>(a);
    else
        spmv_c64_kernel<false><<<(unsigned)grid, kBlock, 0, stream>>>(a);
    DIA_TRY_CUDA(cudaGetLastError());
    return DIA_OK;
}

}  // namespace dia

extern "C" int dia_spmv_rows_c64(int64_t n_rows, int64_t n_cols, int num_diags,
                                 const int* d_offsets, const void* d_vals, int64_t stride,
                                 const void* d_x, void* d_y, cudaStream_t stream)
{
    if (n_rows < 0 || n_cols < 0 || num_diags < 0 || stride < n_rows)
        return fail(DIA_ERR_INVALID, "dia_spmv_rows_c64: bad sizes (stride must be >= n_rows)");
    if (n_rows == 0) return DIA_OK;
    if (!d_y || (num_diags > 0 && (!d_offsets || !d_vals || !d_x)))
        return fail(DIA_ERR_INVALID, "dia_spmv_rows_c64: null pointer");
    if (n_rows + kC64Tile >= (1LL << 31) || n_cols >= (1LL << 31))
        return fail(DIA_ERR_UNSUPPORTED, "dia_spmv_rows_c64: dimensions beyond int32 range");
    SpmvC64Args a{};
    a.vals = (const float2*)d_vals;
    a.x = (const float2*)d_x;
    a.y = (float2*)d_y;
    a.off = d_offsets;
    a.K = num_diags;
    a.n_rows = (int)n_rows;
    a.n_cols = (int)n_cols;
    a.stride = stride;
    return launch_spmv_c64(a, stream);
}

extern "C" int dia_expm_taylor_c64(int64_t n, int num_diags, const int* d_offsets,
                                   const void* d_vals, int64_t stride, float t, int m,
                                   const void* d_x, void* d_y, void* d_work,
                                   cudaStream_t stream)
{
    if (n < 0 || num_diags < 0 || m < 0 || stride < n)
        return fail(DIA_ERR_INVALID, "dia_expm_taylor_c64: bad sizes (stride must be >= n)");
    if (n == 0) return DIA_OK;
    if (!d_x || !d_y || (m > 0 && (!d_work || (num_diags > 0 && (!d_offsets || !d_vals)))))
        return fail(DIA_ERR_INVALID, "dia_expm_taylor_c64: null pointer");
    if (n + kC64Tile >= (1LL << 31))
        return fail(DIA_ERR_UNSUPPORTED, "dia_expm_taylor_c64: n beyond int32 range");
    DIA_TRY_CUDA(cudaMemcpyAsync(d_y, d_x, (size_t)n * 8, cudaMemcpyDeviceToDevice, stream));
    const float2* v = (const float2*)d_x;
    for (int j = 1; j <= m; ++j) {
        float2* vn = (float2*)d_work + (size_t)(j & 1) * (size_t)n;
        SpmvC64Args a{};
        a.vals = (const float2*)d_vals;
        a.x = v;
        a.y = vn;
        a.off = d_offsets;
        a.K = num_diags;
        a.n_rows = (int)n;
        a.n_cols = (int)n;
        a.stride = stride;
        a.c = t / (float)j;
        a.sum = (float2*)d_y;
        const int rc = launch_spmv_c64(a, stream);
        if (rc) return rc;
        v = vn;
    }
    return DIA_OK;
}
