/*
 * dia_oracle.c -- CPU restatement of yuchaosu/DiaGPU's CPU reference paths.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the CUDA
 * library in diagpu_b200/.  Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline leg of bench.py may load it; the library never links it and
 * never falls back to it.
 *
 * Every function restates one reference routine and names the file:line it
 * follows (paths relative to the DiaGPU project root).  Floating-point sums
 * are done in the reference's order with a separate multiply and add; the
 * Makefile builds this file with -ffp-contract=off so that no multiply-add
 * is contracted into an FMA (plain x86-64 g++ -O2, which built the
 * reference's host code, does not contract either).
 *
 * Parity of this restatement is pinned against the reference itself: the
 * Makefile also compiles the reference's own sources into oracle/_ref/
 * (ref_*.cu shims) and tests/golden/make_golden.py records their outputs as
 * fixtures that tests/test_oracle.py replays against these functions.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define ORC_API __attribute__((visibility("default")))

static inline int min0(int x) { return x < 0 ? x : 0; }
static inline int iabs(int x) { return x < 0 ? -x : x; }

/* ------------------------------------------------------------------------
 * SpMV
 * ------------------------------------------------------------------------ */

/* build_recon: spmv/src/dia_reconstruct.cuh:77-107.
 * DIA storage (offsets in any order, value starts, lengths; values of
 * diagonal d start at column max(d,0)) -> K x cols column-indexed Recon with
 * offsets sorted descending.  Recon[k, c] = H[c - d_k, c], zero elsewhere. */
static int cmp_desc(const void* a, const void* b)
{
    int x = *(const int*)a, y = *(const int*)b;
    return (x < y) - (x > y);
}

ORC_API void orc_build_recon(int rows, int cols, int K, const int* offsets,
                             const int* starts, const int* lengths,
                             const float* values, int* out_offsets,
                             float* out_recon)
{
    (void)rows;
    memcpy(out_offsets, offsets, sizeof(int) * (size_t)K);
    qsort(out_offsets, (size_t)K, sizeof(int), cmp_desc);
    memset(out_recon, 0, sizeof(float) * (size_t)K * (size_t)cols);
    for (int k = 0; k < K; ++k) {
        const int d = out_offsets[k];
        int di = -1;                       /* first match, as :92-94 */
        for (int i = 0; i < K; ++i)
            if (offsets[i] == d) { di = i; break; }
        if (di < 0) continue;
        const int sc = d >= 0 ? d : 0;
        for (int j = 0; j < lengths[di]; ++j)
            out_recon[(size_t)k * cols + sc + j] = values[starts[di] + j];
    }
}

/* spmv_from_recon: spmv/test/test_tc_spmv.cu:64-79 (same routine as
 * spmv/test/test_reconstruct.cpp:122-158).  y[r] = sum_k Recon[k, r+d_k] *
 * x[r+d_k], k in storage (descending) order, float accumulator, terms whose
 * column leaves [0, cols) dropped.  x_size bounds the x reads as the GPU
 * launcher's x_size argument does (spmv/src/tc_spmv_regdirect_kernel.cu:
 * 251-257); pass x_size == cols for the CPU routine's behaviour. */
ORC_API void orc_spmv_recon(int rows, int cols, int K, const int* offsets,
                            const float* recon, const float* x, int x_size,
                            float* y)
{
    const int xe = x_size < cols ? x_size : cols;
    for (int r = 0; r < rows; ++r) {
        float s = 0.0f;
        for (int k = 0; k < K; ++k) {
            const long c = (long)r + offsets[k];
            if (c >= 0 && c < xe) {
                const float p = recon[(size_t)k * cols + c] * x[c];
                s = s + p;
            }
        }
        y[r] = s;
    }
}

/* CPU CSR reference: spmv/bench/bench_cusparse.cu:119-126 (serial float
 * accumulation over each row's columns in ascending order). */
ORC_API void orc_spmv_csr(int n, const int* rowptr, const int* colidx,
                          const float* vals, const float* x, float* y)
{
    for (int r = 0; r < n; ++r) {
        float s = 0.0f;
        for (int p = rowptr[r]; p < rowptr[r + 1]; ++p) {
            const float t = vals[p] * x[colidx[p]];
            s = s + t;
        }
        y[r] = s;
    }
}

/* The same sum on the library's row-indexed padded layout:
 * vals[k*stride + i] = A[row0+i, row0+i+d_k].  Rows [0, nrows) of the block
 * starting at global row row0; x holds global columns [x_lo, x_lo+x_len).
 * Order: k = 0..K-1 as stored (ascending offsets reproduce the CSR loop
 * above, descending offsets reproduce spmv_from_recon). */
ORC_API void orc_spmv_rowidx(int64_t row0, int64_t nrows, int64_t ncols,
                             int K, const int* offsets, const float* vals,
                             int64_t stride, const float* x, int64_t x_lo,
                             int64_t x_len, float* y, int threads)
{
    (void)threads;
#pragma omp parallel for schedule(static) num_threads(threads > 0 ? threads : 1)
    for (int64_t i = 0; i < nrows; ++i) {
        const int64_t g = row0 + i;
        float s = 0.0f;
        for (int k = 0; k < K; ++k) {
            const int64_t c = g + offsets[k];
            if (c < 0 || c >= ncols || c < x_lo || c >= x_lo + x_len) continue;
            const float p = vals[(size_t)k * stride + i] * x[c - x_lo];
            s = s + p;
        }
        y[i] = s;
    }
}

/* Truncated Taylor series of exp(tA) x (the library's dia_expm_taylor): the
 * reference has no such driver, so this is the definition the library
 * follows, built from the SpMV loop above: v_0 = x, v_j = fl(t/j) * (A
 * v_{j-1}) rounded per element, y = ((v_0 + v_1) + v_2) + ... element by
 * element.  A is a whole square matrix on the row-indexed layout. */
ORC_API void orc_expm_taylor(int64_t n, int K, const int* offsets, const float* vals,
                             int64_t stride, float t, int m, const float* x, float* y,
                             int threads)
{
    float* v = (float*)malloc((size_t)n * sizeof(float));
    float* w = (float*)malloc((size_t)n * sizeof(float));
    memcpy(v, x, (size_t)n * sizeof(float));
    memcpy(y, x, (size_t)n * sizeof(float));
    for (int j = 1; j <= m; ++j) {
        const float c = t / (float)j;
        orc_spmv_rowidx(0, n, n, K, offsets, vals, stride, v, 0, n, w, threads);
#pragma omp parallel for schedule(static) num_threads(threads > 0 ? threads : 1)
        for (int64_t i = 0; i < n; ++i) {
            const float q = c * w[i];
            w[i] = q;
            y[i] = y[i] + q;
        }
        float* tmp = v;
        v = w;
        w = tmp;
    }
    free(v);
    free(w);
}

/* Lanczos on a symmetric DIA operator (the library's dia_lanczos): the
 * reference has no eigensolver, so this is the definition the library
 * follows.  fp32 vector updates in the order below, fp64 dot products of
 * exact fp32 products (summed sequentially here; the library sums the same
 * exact products in a fixed tree, agreeing to ~1e-16 relative), scalars
 * rounded to fp32 where the vectors use them. */
ORC_API void orc_lanczos(int64_t n, int K, const int* offsets, const float* vals, int64_t stride,
                         int m, const float* x, double* alpha, double* beta, float* basis)
{
    float* v = (float*)malloc((size_t)n * sizeof(float));
    float* vp = (float*)calloc((size_t)n, sizeof(float));
    float* w = (float*)malloc((size_t)n * sizeof(float));
    double ss = 0.0;
    for (int64_t i = 0; i < n; ++i) ss += (double)x[i] * (double)x[i];
    float inv = 1.0f / (float)sqrt(ss);
    for (int64_t i = 0; i < n; ++i) v[i] = x[i] * inv;
    for (int j = 0; j < m; ++j) {
        if (basis) memcpy(basis + (size_t)j * n, v, (size_t)n * sizeof(float));
        const float bp = j ? (float)beta[j - 1] : 0.0f;
        double dot = 0.0;
        for (int64_t i = 0; i < n; ++i) {
            float s = 0.0f;
            for (int k = 0; k < K; ++k) {
                const int64_t c = i + offsets[k];
                if (c < 0 || c >= n) continue;
                const float p = vals[(size_t)k * stride + i] * v[c];
                s = s + p;
            }
            if (j) {
                const float q = bp * vp[i];
                s = s - q;
            }
            w[i] = s;
            dot += (double)s * (double)v[i];
        }
        alpha[j] = dot;
        const float al = (float)dot;
        ss = 0.0;
        for (int64_t i = 0; i < n; ++i) {
            const float q = al * v[i];
            w[i] = w[i] - q;
            ss += (double)w[i] * (double)w[i];
        }
        beta[j] = sqrt(ss);
        inv = 1.0f / (float)beta[j];
        float* t = vp;
        vp = v;
        v = t;
        for (int64_t i = 0; i < n; ++i) v[i] = w[i] * inv;
    }
    free(v);
    free(vp);
    free(w);
}

/* Complex64 SpMV on the row-indexed layout (the library's
 * dia_spmv_rows_c64; the reference is real-only): values and x interleaved
 * (re, im); per term re += fl(fl(ar*xr) - fl(ai*xi)), im += fl(fl(ar*xi) +
 * fl(ai*xr)), terms in offset storage order, whole square or rectangular
 * matrix. */
ORC_API void orc_spmv_rowidx_c64(int64_t nrows, int64_t ncols, int K, const int* offsets,
                                 const float* vals, int64_t stride, const float* x, float* y,
                                 int threads)
{
    (void)threads;
#pragma omp parallel for schedule(static) num_threads(threads > 0 ? threads : 1)
    for (int64_t i = 0; i < nrows; ++i) {
        float sr = 0.0f, si = 0.0f;
        for (int k = 0; k < K; ++k) {
            const int64_t c = i + offsets[k];
            if (c < 0 || c >= ncols) continue;
            const float ar = vals[2 * ((size_t)k * stride + i)];
            const float ai = vals[2 * ((size_t)k * stride + i) + 1];
            const float xr = x[2 * c], xi = x[2 * c + 1];
            const float p1 = ar * xr, p2 = ai * xi, p3 = ar * xi, p4 = ai * xr;
            const float pr = p1 - p2, pi = p3 + p4;
            sr = sr + pr;
            si = si + pi;
        }
        y[2 * i] = sr;
        y[2 * i + 1] = si;
    }
}

/* exp(-i t A) x by the truncated Taylor series (dia_expm_taylor_c64):
 * v_0 = x, v_j = (-i c_j) (A v_{j-1}) with c_j = fl(t/j), i.e.
 * (re, im) = (fl(c_j * s_im), -fl(c_j * s_re)); y = y + v_j per element. */
ORC_API void orc_expm_taylor_c64(int64_t n, int K, const int* offsets, const float* vals,
                                 int64_t stride, float t, int m, const float* x, float* y,
                                 int threads)
{
    float* v = (float*)malloc((size_t)n * 2 * sizeof(float));
    float* w = (float*)malloc((size_t)n * 2 * sizeof(float));
    memcpy(v, x, (size_t)n * 2 * sizeof(float));
    memcpy(y, x, (size_t)n * 2 * sizeof(float));
    for (int j = 1; j <= m; ++j) {
        const float c = t / (float)j;
        orc_spmv_rowidx_c64(n, n, K, offsets, vals, stride, v, w, threads);
#pragma omp parallel for schedule(static) num_threads(threads > 0 ? threads : 1)
        for (int64_t i = 0; i < n; ++i) {
            const float re = c * w[2 * i + 1];
            const float im = -(c * w[2 * i]);
            w[2 * i] = re;
            w[2 * i + 1] = im;
            y[2 * i] = y[2 * i] + re;
            y[2 * i + 1] = y[2 * i + 1] + im;
        }
        float* tmp = v;
        v = w;
        w = tmp;
    }
    free(v);
    free(w);
}

/* ------------------------------------------------------------------------
 * SpMSpM symbolic phase
 * ------------------------------------------------------------------------ */

/* make_c_structure: spmspm/bench_spmspm.cu:109-131 (also
 * compute_c_hm_structure, spmspm/paper_hm.cuh:87-117, and the k-set of
 * build_c_layout, gemm_diag/gemm_diag.cu:387-423).  Output offsets are the
 * ascending set {da + db : -n < da + db < n}; lengths n - |d|; starts are the
 * prefix sums of the lengths.  Returns the number of C diagonals.  Any
 * output pointer may be NULL (count only). */
ORC_API int orc_c_structure(int n, const int* A_off, int nA, const int* B_off,
                            int nB, int* C_off, int* C_len, int64_t* C_start)
{
    if (n <= 0) return 0;
    char* present = (char*)calloc((size_t)2 * n - 1, 1);
    for (int a = 0; a < nA; ++a)
        for (int b = 0; b < nB; ++b) {
            const long dc = (long)A_off[a] + B_off[b];
            if (dc > -(long)n && dc < (long)n) present[dc + (n - 1)] = 1;
        }
    int nC = 0;
    int64_t off = 0;
    for (long d = -(long)(n - 1); d <= (long)(n - 1); ++d) {
        if (!present[d + (n - 1)]) continue;
        const int len = n - iabs((int)d);
        if (len <= 0) continue;
        if (C_off) C_off[nC] = (int)d;
        if (C_len) C_len[nC] = len;
        if (C_start) C_start[nC] = off;
        off += len;
        ++nC;
    }
    free(present);
    return nC;
}

/* Pair lists per C diagonal in the order cpu_dia_spgemm visits them
 * (spmspm/bench_spmspm.cu:392-397: A diagonals in storage order, B found by
 * offset; the last B diagonal of a repeated offset wins, as its
 * unordered_map assignment at :379 does).  pair_ptr has nC+1 entries; the
 * pair arrays are sized by the return value of a first call with NULLs. */
ORC_API int64_t orc_pair_lists(int n, const int* A_off, int nA,
                               const int* B_off, int nB, const int* C_off,
                               int nC, int* pair_ptr, int* pair_a, int* pair_b)
{
    int64_t np = 0;
    for (int k = 0; k < nC; ++k) {
        if (pair_ptr) pair_ptr[k] = (int)np;
        for (int a = 0; a < nA; ++a) {
            const long db = (long)C_off[k] - A_off[a];
            int bi = -1;
            for (int b = 0; b < nB; ++b)
                if (B_off[b] == db) bi = b;
            if (bi < 0) continue;
            (void)n;
            if (pair_a) pair_a[np] = a;
            if (pair_b) pair_b[np] = bi;
            ++np;
        }
    }
    if (pair_ptr) pair_ptr[nC] = (int)np;
    return np;
}

/* ------------------------------------------------------------------------
 * SpMSpM numeric phase (HM layout: diagonal d stored from position
 * min(row, col) = row + min(d, 0), length n - |d|)
 * ------------------------------------------------------------------------ */

static int find_b(const int* B_off, int nB, int db)
{
    int bi = -1;
    for (int b = 0; b < nB; ++b)
        if (B_off[b] == db) bi = b;
    return bi;
}

/* cpu_dia_spgemm: spmspm/bench_spmspm.cu:376-408.  For every C diagonal and
 * position p, acc = sum over A diagonals (storage order) of
 * A[pa] * B[pb] with pa = p + min0(da) - min0(dc),
 * pb = p + da + min0(db) - min0(dc), terms outside either diagonal dropped;
 * float accumulator starting at 0.  Parallel over C diagonals (OpenMP,
 * dynamic) exactly as the reference; the per-element order is sequential, so
 * the result does not depend on the thread count. */
ORC_API void orc_dia_spgemm_hm(int n,
                               const int* A_off, const int* A_len,
                               const int64_t* A_start, const float* A_val,
                               int nA,
                               const int* B_off, const int* B_len,
                               const int64_t* B_start, const float* B_val,
                               int nB,
                               const int* C_off, const int* C_len,
                               const int64_t* C_start, int nC, float* C_val,
                               int threads)
{
    (void)n;
    int* bmap = (int*)malloc(sizeof(int) * (size_t)(nA > 0 ? nA : 1) *
                             (size_t)(nC > 0 ? nC : 1));
    for (int k = 0; k < nC; ++k)
        for (int a = 0; a < nA; ++a)
            bmap[(size_t)k * nA + a] =
                find_b(B_off, nB, C_off[k] - A_off[a]);
#pragma omp parallel for schedule(dynamic) num_threads(threads > 0 ? threads : 1)
    for (int k = 0; k < nC; ++k) {
        const int dc = C_off[k];
        const int minc = min0(dc);
        for (int p = 0; p < C_len[k]; ++p) {
            float acc = 0.0f;
            for (int a = 0; a < nA; ++a) {
                const int bi = bmap[(size_t)k * nA + a];
                if (bi < 0) continue;
                const int da = A_off[a];
                const int db = dc - da;
                const long pa = (long)p + min0(da) - minc;
                const long pb = (long)p + da + min0(db) - minc;
                if (pa < 0 || pa >= A_len[a]) continue;
                if (pb < 0 || pb >= B_len[bi]) continue;
                const float t = A_val[A_start[a] + pa] * B_val[B_start[bi] + pb];
                acc = acc + t;
            }
            C_val[C_start[k] + p] = acc;
        }
    }
    free(bmap);
}

/* The same sum accumulated in double: the reference value for the TF32
 * tolerance check of the dense-band path and for separating summation-order
 * noise from real errors. */
ORC_API void orc_dia_spgemm_hm_f64(int n,
                                   const int* A_off, const int* A_len,
                                   const int64_t* A_start, const float* A_val,
                                   int nA,
                                   const int* B_off, const int* B_len,
                                   const int64_t* B_start, const float* B_val,
                                   int nB,
                                   const int* C_off, const int* C_len,
                                   const int64_t* C_start, int nC,
                                   double* C_val, int threads)
{
    (void)n;
#pragma omp parallel for schedule(dynamic) num_threads(threads > 0 ? threads : 1)
    for (int k = 0; k < nC; ++k) {
        const int dc = C_off[k];
        const int minc = min0(dc);
        int* bi_of = (int*)malloc(sizeof(int) * (size_t)(nA > 0 ? nA : 1));
        for (int a = 0; a < nA; ++a) bi_of[a] = find_b(B_off, nB, dc - A_off[a]);
        for (int p = 0; p < C_len[k]; ++p) {
            double acc = 0.0;
            for (int a = 0; a < nA; ++a) {
                const int bi = bi_of[a];
                if (bi < 0) continue;
                const int da = A_off[a];
                const int db = dc - da;
                const long pa = (long)p + min0(da) - minc;
                const long pb = (long)p + da + min0(db) - minc;
                if (pa < 0 || pa >= A_len[a]) continue;
                if (pb < 0 || pb >= B_len[bi]) continue;
                acc += (double)A_val[A_start[a] + pa] *
                       (double)B_val[B_start[bi] + pb];
            }
            C_val[C_start[k] + p] = acc;
        }
        free(bi_of);
    }
}

/* ------------------------------------------------------------------------
 * gemm_diag (row-packed inputs DA[ri*n + row], HM-packed output)
 * ------------------------------------------------------------------------ */

/* build_c_layout: gemm_diag/gemm_diag.cu:387-423.  C_offsets are VALUE
 * starts (int), C_lens = n - |k|, k_to_idx[k + n-1] = index or -1, k_list =
 * the ascending diagonal offsets.  Returns num_k; *total_c receives the
 * value count. */
ORC_API int orc_build_c_layout(int n, const int* off_A, int P,
                               const int* off_B, int Q, int* C_offsets,
                               int* C_lens, int* k_to_idx, int* k_list,
                               int64_t* total_c)
{
    char* present = (char*)calloc((size_t)2 * n - 1, 1);
    for (int i = 0; i < P; ++i)
        for (int j = 0; j < Q; ++j) {
            const long k = (long)off_A[i] + off_B[j];
            if (k >= -(long)(n - 1) && k <= (long)(n - 1))
                present[k + (n - 1)] = 1;
        }
    int num_k = 0;
    int64_t tot = 0;
    for (long k = -(long)(n - 1); k <= (long)(n - 1); ++k) {
        if (k_to_idx) k_to_idx[k + (n - 1)] = -1;
        if (!present[k + (n - 1)]) continue;
        const int len = n - iabs((int)k);
        if (len <= 0) continue;
        if (k_to_idx) k_to_idx[k + (n - 1)] = num_k;
        if (k_list) k_list[num_k] = (int)k;
        if (C_offsets) C_offsets[num_k] = (int)tot;
        if (C_lens) C_lens[num_k] = len;
        tot += len;
        ++num_k;
    }
    free(present);
    if (total_c) *total_c = tot;
    return num_k;
}

/* cpu_diag_multiply: gemm_diag/gemm_diag.cu:334-356, written into the
 * HM-packed C instead of a dense n x n matrix.  For every (ri, rj) in that
 * order and row t: a = DA[ri][t], b = DB[rj][t + i]; zero a or b skipped;
 * C[row t, col t+i+j] += a*b in float.  Output is accumulated into C_data
 * (the caller zeroes it, as the reference memsets before its kernel). */
ORC_API void orc_gemm_diag_f32(const float* DA, const int* off_A, int P,
                               const float* DB, const int* off_B, int Q, int n,
                               float* C_data, const int* C_offsets,
                               const int* k_to_idx)
{
    for (int ri = 0; ri < P; ++ri) {
        const int i = off_A[ri];
        for (int rj = 0; rj < Q; ++rj) {
            const int j = off_B[rj];
            for (int t = 0; t < n; ++t) {
                const float a = DA[(size_t)ri * n + t];
                const long bt = (long)t + i;
                if (bt < 0 || bt >= n) continue;
                const float b = DB[(size_t)rj * n + bt];
                if (a == 0.0f || b == 0.0f) continue;
                const long col = (long)t + i + j;
                if (col < 0 || col >= n) continue;
                const int k = i + j;
                const int ki = k_to_idx[k + (n - 1)];
                if (ki < 0) continue;
                const long p = (long)t + min0(k);      /* row - c_sr */
                const float prod = a * b;
                float* c = &C_data[(size_t)C_offsets[ki] + p];
                *c = *c + prod;
            }
        }
    }
}

/* The same product accumulated in double over the (ri, rj) pairs, the
 * reference for the TF32 tolerance check at sizes where the dense n x n
 * routine cannot run (gemm_diag/gemm_diag.cu:497-502 limits it to n<=4096).
 * Parallel over output rows. */
ORC_API void orc_gemm_diag_f64(const float* DA, const int* off_A, int P,
                               const float* DB, const int* off_B, int Q, int n,
                               double* C_data, const int* C_offsets,
                               const int* k_to_idx, int threads)
{
#pragma omp parallel for schedule(static) num_threads(threads > 0 ? threads : 1)
    for (int t = 0; t < n; ++t) {
        for (int ri = 0; ri < P; ++ri) {
            const int i = off_A[ri];
            const double a = DA[(size_t)ri * n + t];
            const long bt = (long)t + i;
            if (bt < 0 || bt >= n || a == 0.0) continue;
            for (int rj = 0; rj < Q; ++rj) {
                const int j = off_B[rj];
                const long col = (long)t + i + j;
                if (col < 0 || col >= n) continue;
                const int ki = k_to_idx[i + j + (n - 1)];
                if (ki < 0) continue;
                const double b = DB[(size_t)rj * n + bt];
                C_data[(size_t)C_offsets[ki] + t + min0(i + j)] += a * b;
            }
        }
    }
}

/* ------------------------------------------------------------------------
 * Synthetic inputs (the library's own generator, restated here so the GPU
 * generator can be checked bit for bit).  Not a reference routine: the
 * reference seeds std::mt19937 / an LCG / integer hashes per program; the
 * B200 build needs a generator any rank can evaluate for any (offset, row)
 * independently, so values are a counter-based hash of (seed, offset, row).
 * ------------------------------------------------------------------------ */

static inline uint64_t mix64(uint64_t z)
{
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

static inline uint64_t key3(uint64_t seed, int32_t d, int64_t row)
{
    return mix64(mix64(seed ^ ((uint64_t)(uint32_t)d * 0xD6E8FEB86659FD93ull)) ^
                 (uint64_t)row);
}

/* kind 0: base + lo + (hi-lo)*u, u = top 24 hash bits / 2^24.
 * kind 1: base + scale * IrwinHall12 (sum of 12 such u minus 6; mean 0,
 *         variance 1), computed in integers then converted once. */
static inline float synth_value(uint64_t seed, int32_t d, int64_t row, int kind,
                                float base, float lo, float hi)
{
    uint64_t h = key3(seed, d, row);
    if (kind == 0) {
        const float u = (float)(uint32_t)(h >> 40) * (1.0f / 16777216.0f);
        const float w = hi - lo;
        const float t = w * u;
        const float v = lo + t;
        return base + v;
    }
    int64_t s = 0;
    for (int r = 0; r < 12; ++r) {
        s += (int64_t)(h >> 40);
        h = mix64(h);
    }
    s -= (int64_t)6 * 16777216;
    const float z = (float)s * (1.0f / 16777216.0f);
    const float t = hi * z;          /* hi carries the scale for kind 1 */
    return base + t;
}

/* Fill rows [row0, row0+nrows) of a matrix in the padded row-indexed layout
 * (vals[k*stride + i], zero where row or column is out of range, zero in
 * the stride padding).  base[k] is added to every value of diagonal k. */
ORC_API void orc_synth_rowidx(uint64_t seed, int64_t n_rows, int64_t n_cols,
                              int K, const int* offsets, const float* base,
                              int kind, float lo, float hi, int64_t row0,
                              int64_t nrows, int64_t stride, float* vals)
{
    for (int k = 0; k < K; ++k)
        for (int64_t i = 0; i < stride; ++i) {
            const int64_t g = row0 + i;
            const int64_t c = g + offsets[k];
            float v = 0.0f;
            if (i < nrows && g < n_rows && c >= 0 && c < n_cols)
                v = synth_value(seed, offsets[k], g, kind, base ? base[k] : 0.0f,
                                lo, hi);
            vals[(size_t)k * stride + i] = v;
        }
}

ORC_API void orc_synth_vector(uint64_t seed, int64_t i0, int64_t len,
                              float lo, float hi, float* out)
{
    for (int64_t i = 0; i < len; ++i)
        out[i] = synth_value(seed, 0x7fffffff, i0 + i, 0, 0.0f, lo, hi);
}
