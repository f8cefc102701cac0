/*
 * krylov.cu -- Lanczos on a DIA operator, entirely on the device.
 *
 * For a symmetric A (a Hamiltonian, a Laplacian) m Lanczos steps build the
 * tridiagonal T_m = tridiag(beta, alpha, beta) whose extreme eigenvalues
 * approach A's (ground-state energies); together with the Taylor driver in
 * spmv.cu this is the chain of SpMVs the reference's operators are built
 * for -- the reference itself stops at single products.  One step j:
 *     w      = fl(A v_j) - fl(beta_{j-1} * v_{j-1})      (SpMV fused, + alpha partials)
 *     alpha_j = sum_i w_i * v_j,i                        (fp64, fixed-order tree)
 *     w      = w - fl(alpha_j * v_j)                     (+ beta partials)
 *     beta_j = sqrt(sum_i w_i^2)                         (fp64, fixed-order tree)
 *     v_{j+1} = fl(w * fl(1 / beta_j))
 * with alpha_j and beta_j kept in device memory (fp64) and used by the
 * vector updates as fp32, so m steps run without any host synchronisation.
 * Products of two fp32 values are exact in fp64, so the fp64 dot products
 * agree with any other summation order to about 1e-16 relative; the fp32
 * vector updates follow the order above, which the CPU oracle restates.
 * The starting vector is normalised the same way (v_0 = x * fl(1/||x||)).
 */
#include <cmath>

#include "../../include/diagpu_b200.h"
#include "dia_core.cuh"

namespace dia {

constexpr int kKrThreads = 256;
constexpr int kKrRows = kKrThreads * 4;   /* rows per CTA */

/* fixed-order CTA reduction of one fp64 value per thread */
__device__ __forceinline__ double block_sum(double v)
{
    __shared__ double s[kKrThreads / 32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) v += __shfl_down_sync(0xffffffffu, v, d);
    if (lane == 0) s[warp] = v;
    __syncthreads();
    double t = 0.0;
    if (threadIdx.x == 0)
        for (int w = 0; w < kKrThreads / 32; ++w) t += s[w];
    __syncthreads();
    return t;   /* valid in thread 0 */
}

struct KrArgs {
    const float* vals;
    const int* off;
    int K, n;
    long long stride;
};

/* sum of part[0..nb) in the reduce kernel's fixed order, in every thread
 * of the CTA: each CTA of a consumer kernel repeats it and gets the same
 * bits, which saves the single-CTA reduce launch between two vector
 * kernels (nb doubles, a few KB, come from L2) */
__device__ __forceinline__ double all_sum(const double* __restrict__ part, int nb)
{
    __shared__ double s_t;
    double acc = 0.0;
    for (int b = threadIdx.x; b < nb; b += kKrThreads) acc += part[b];
    const double t = block_sum(acc);
    if (threadIdx.x == 0) s_t = t;
    __syncthreads();
    return s_t;
}

/* One Lanczos step's SpMV with the previous step's scaling fused in:
 *     beta = sqrt(sum of part_in)  (every CTA, fixed order; CTA 0 records it
 *            in beta_rec unless null),  inv = fl(1 / beta),
 *     v[c] = fl(wsrc[c] * inv)     (computed wherever the SpMV reads it; the
 *            CTA's own rows are stored in v_out),
 *     w    = fl(A v) - fl(beta * v_prev)   (no v_prev in the first step),
 *     part_out[b] = sum over the CTA's rows of w * v.
 * The first step scales x by its norm the same way. */
template <bool CACHE>
__global__ void __launch_bounds__(kKrThreads)
lanczos_spmv_kernel(KrArgs a, const float* __restrict__ wsrc, const double* __restrict__ part_in,
                    int nb, double* __restrict__ beta_rec, const float* __restrict__ v_prev,
                    float* __restrict__ v_out, float* __restrict__ w, double* __restrict__ part)
{
    __shared__ int s_off[kMaxTerms];
    const int K = min(a.K, kMaxTerms);
    for (int k = threadIdx.x; k < K; k += kKrThreads) s_off[k] = a.off[k];
    const double bd = sqrt(all_sum(part_in, nb));   /* synchronises s_off too */
    if (beta_rec && blockIdx.x == 0 && threadIdx.x == 0) *beta_rec = bd;
    const float inv = __frcp_rn((float)bd);
    const float bp = (float)bd;
    double dot = 0.0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const int i = blockIdx.x * kKrRows + j * kKrThreads + threadIdx.x;
        if (i >= a.n) continue;
        float s = 0.0f;
        for (int k = 0; k < K; ++k) {
            const int c = i + s_off[k];
            if (c < 0 || c >= a.n) continue;
            const float* vp = a.vals + (long long)k * a.stride + i;
            s = __fadd_rn(s, __fmul_rn(CACHE ? __ldg(vp) : __ldcs(vp),
                                       __fmul_rn(__ldg(wsrc + c), inv)));
        }
        const float vi = __fmul_rn(wsrc[i], inv);
        v_out[i] = vi;
        const float wi = v_prev ? __fsub_rn(s, __fmul_rn(bp, v_prev[i])) : s;
        w[i] = wi;
        dot += (double)wi * (double)vi;
    }
    const double t = block_sum(dot);
    if (threadIdx.x == 0) part[blockIdx.x] = t;
}

/* one CTA: out = sum of part[0..nb) in a fixed order, sqrt when asked */
__global__ void __launch_bounds__(kKrThreads)
lanczos_reduce_kernel(const double* __restrict__ part, int nb, double* __restrict__ out, int root)
{
    double acc = 0.0;
    for (int b = threadIdx.x; b < nb; b += kKrThreads) acc += part[b];
    const double t = block_sum(acc);
    if (threadIdx.x == 0) *out = root ? sqrt(t) : t;
}

/* alpha = sum of the SpMV's partials (CTA 0 records it); w = w -
 * fl(alpha * v); part_out[b] = sum of w^2 */
__global__ void __launch_bounds__(kKrThreads)
lanczos_orth_kernel(int n, const float* __restrict__ v, const double* __restrict__ part_in,
                    int nb, double* __restrict__ alpha, float* __restrict__ w,
                    double* __restrict__ part_out)
{
    const double ad = all_sum(part_in, nb);
    if (blockIdx.x == 0 && threadIdx.x == 0) *alpha = ad;
    const float al = (float)ad;
    double ss = 0.0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const int i = blockIdx.x * kKrRows + j * kKrThreads + threadIdx.x;
        if (i >= n) continue;
        const float wi = __fsub_rn(w[i], __fmul_rn(al, v[i]));
        w[i] = wi;
        ss += (double)wi * (double)wi;
    }
    const double t = block_sum(ss);
    if (threadIdx.x == 0) part_out[blockIdx.x] = t;
}

/* part[b] = sum of x^2 over the CTA's rows (x is only read) */
__global__ void __launch_bounds__(kKrThreads)
lanczos_norm_kernel(int n, const float* __restrict__ x, double* __restrict__ part)
{
    double ss = 0.0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const int i = blockIdx.x * kKrRows + j * kKrThreads + threadIdx.x;
        if (i < n) ss += (double)x[i] * (double)x[i];
    }
    const double t = block_sum(ss);
    if (threadIdx.x == 0) part[blockIdx.x] = t;
}

}  // namespace dia

using namespace dia;

extern "C" int64_t dia_lanczos_workspace(int64_t n)
{
    if (n <= 0) return -1;
    const int64_t nb = (n + kKrRows - 1) / kKrRows;
    return 4 * n * 4 + 2 * nb * 8 + 64;
}

extern "C" int dia_lanczos(int64_t n, int num_diags, const int* d_offsets, const float* d_vals,
                           int64_t stride, int m, const float* d_x, double* d_alpha,
                           double* d_beta, float* d_basis, void* d_work, int64_t work_bytes,
                           cudaStream_t stream)
{
    if (n <= 0 || num_diags < 0 || m < 0 || stride < n)
        return fail(DIA_ERR_INVALID, "dia_lanczos: bad sizes (stride must be >= n)");
    if (num_diags > kMaxTerms)
        return fail(DIA_ERR_UNSUPPORTED, "dia_lanczos: more diagonals than one CTA stages");
    if (n + kKrRows >= (1LL << 31))
        return fail(DIA_ERR_UNSUPPORTED, "dia_lanczos: n beyond int32 range");
    if (!d_x || !d_alpha || !d_beta || !d_work || (num_diags > 0 && (!d_offsets || !d_vals)))
        return fail(DIA_ERR_INVALID, "dia_lanczos: null pointer");
    if (work_bytes < dia_lanczos_workspace(n))
        return fail(DIA_ERR_INVALID, "dia_lanczos: workspace smaller than dia_lanczos_workspace()");
    const int nb = (int)((n + kKrRows - 1) / kKrRows);
    float* w = (float*)d_work;
    float* wbuf[2] = {w, w + n};
    float* vbuf[2] = {w + 2 * n, w + 3 * n};
    /* two partial-sum buffers: a kernel that reduces one writes the other */
    double* part = (double*)(((uintptr_t)(w + 4 * n) + 7) & ~(uintptr_t)7);
    double* part2 = part + nb;
    KrArgs a{d_vals, d_offsets, num_diags, (int)n, stride};
    /* every step reads the whole matrix: when its values fit in about half
     * of L2 they are read with normal caching and stay there across steps;
     * larger operators stream (evict-first) */
    const bool cache = (long long)num_diags * stride * 4 <= (48LL << 20);
    /* ||x||^2 partials; the first SpMV scales x by the norm */
    lanczos_norm_kernel<<<nb, kKrThreads, 0, stream>>>((int)n, d_x, part2);
    DIA_TRY_CUDA(cudaGetLastError());
    /* two launches per step: SpMV (the previous step's scaling fused in,
     * + alpha partials) and orthogonalise (alpha reduced in every CTA,
     * + beta partials); the last beta is reduced in one CTA.  The SpMV reads
     * the previous w while writing the new one, so w alternates between two
     * buffers (and v with it) */
    for (int j = 0; j < m; ++j) {
        float* v = vbuf[j & 1];
        float* vp = vbuf[(j + 1) & 1];
        float* wj = wbuf[j & 1];
        const float* wsrc = j ? wbuf[(j + 1) & 1] : d_x;
        if (cache)
            lanczos_spmv_kernel<true><<<nb, kKrThreads, 0, stream>>>(
                a, wsrc, part2, nb, j ? d_beta + j - 1 : nullptr, j ? vp : nullptr, v, wj, part);
        else
            lanczos_spmv_kernel<false><<<nb, kKrThreads, 0, stream>>>(
                a, wsrc, part2, nb, j ? d_beta + j - 1 : nullptr, j ? vp : nullptr, v, wj, part);
        DIA_TRY_CUDA(cudaGetLastError());
        if (d_basis)
            DIA_TRY_CUDA(cudaMemcpyAsync(d_basis + (size_t)j * n, v, (size_t)n * 4,
                                         cudaMemcpyDeviceToDevice, stream));
        lanczos_orth_kernel<<<nb, kKrThreads, 0, stream>>>((int)n, v, part, nb, d_alpha + j, wj,
                                                          part2);
        DIA_TRY_CUDA(cudaGetLastError());
    }
    if (m > 0) {
        lanczos_reduce_kernel<<<1, kKrThreads, 0, stream>>>(part2, nb, d_beta + m - 1, 1);
        DIA_TRY_CUDA(cudaGetLastError());
    }
    return DIA_OK;
}
