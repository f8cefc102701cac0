/*
 * chain.cu -- device-side symbolic phase and product for matrix-power chains.
 *
 * In a chain P_{k+1} = P_k * H (H narrow, P_k filling in step by step), the
 * host symbolic phase and plan upload of every step would need P_k's offset
 * set on the host, i.e. one synchronisation per step; the reference notes
 * that this host rebuild dominates the sub-millisecond product
 * (spmspm/gather_flat.cuh:13-14, 110-117) and resolves pairs on the device,
 * but still takes the output offsets from the host.  Here the whole step
 * stays on the device:
 *   sumset_mark_kernel   -- every (a, b) pair sets bit a+b+n-1 of a bitmap
 *                           over the 2n-1 possible offsets;
 *   sumset_count_kernel  -- population count per 1024-word block;
 *   sumset_scan_kernel   -- one CTA scans the block counts; the total is the
 *                           output diagonal count (written to device memory);
 *   sumset_write_kernel  -- every set bit writes its offset at its rank, so
 *                           the offsets come out ascending -- the order of the
 *                           reference's make_c_structure
 *                           (spmspm/bench_spmspm.cu:109-131), bit for bit;
 * then the generic path's device pair resolution (pair_plan_kernel, in A
 * storage order) and pair-sum kernel run with their counts read on the
 * device.  Nothing is copied to the host; a count above the caller's
 * capacity is reported by the stored count itself (the product then holds
 * only the first nC_cap diagonals and must not be used).
 */
#include <algorithm>

#include "../../include/diagpu_b200.h"
#include "dia_core.cuh"

namespace dia {

constexpr int kScanThreads = 256;
constexpr int kWordsPerThread = 4;
constexpr int kWordsPerBlock = kScanThreads * kWordsPerThread;

struct ChainWork {
    unsigned* bitmap;
    int* block_sums;
    Term* terms;
    OutDesc* outs;
    long long nwords, nblocks;
    size_t bytes;
};

static size_t align256(size_t x) { return (x + 255) / 256 * 256; }

static ChainWork chain_layout(void* base, long long n, int nA_cap, int nC_cap)
{
    ChainWork w{};
    w.nwords = (2 * n - 1 + 31) / 32;
    w.nblocks = (w.nwords + kWordsPerBlock - 1) / kWordsPerBlock;
    const size_t b_bitmap = align256((size_t)w.nwords * 4);
    const size_t b_sums = align256((size_t)w.nblocks * 4);
    const size_t b_terms = align256((size_t)nC_cap * std::max(nA_cap, 1) * sizeof(Term));
    const size_t b_outs = align256((size_t)nC_cap * sizeof(OutDesc));
    char* p = (char*)base;
    w.bitmap = (unsigned*)p;
    w.block_sums = (int*)(p + b_bitmap);
    w.terms = (Term*)(p + b_bitmap + b_sums);
    w.outs = (OutDesc*)(p + b_bitmap + b_sums + b_terms);
    w.bytes = b_bitmap + b_sums + b_terms + b_outs;
    return w;
}

__global__ void sumset_mark_kernel(const int* __restrict__ A_off, const int* __restrict__ nA_dev,
                                   int nA_cap, const int* __restrict__ B_off, int nB, int n,
                                   unsigned* __restrict__ bitmap)
{
    const int nA = min(*nA_dev, nA_cap);
    const long long total = (long long)nA * nB;
    for (long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x; t < total;
         t += (long long)gridDim.x * blockDim.x) {
        const long long c = (long long)A_off[t / nB] + B_off[t % nB];
        if (c > -n && c < n) {
            const long long bit = c + n - 1;
            atomicOr(&bitmap[bit >> 5], 1u << (bit & 31));
        }
    }
}

/* exclusive scan of one value per thread over the CTA; returns the total */
__device__ __forceinline__ int block_exclusive_scan(int v, int& total)
{
    __shared__ int s_warp[kScanThreads / 32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int x = v;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, x, d);
        if (lane >= d) x += y;
    }
    if (lane == 31) s_warp[warp] = x;
    __syncthreads();
    int before = 0;
    total = 0;
    for (int w = 0; w < kScanThreads / 32; ++w) {
        before += w < warp ? s_warp[w] : 0;
        total += s_warp[w];
    }
    __syncthreads();
    return before + x - v;
}

__global__ void __launch_bounds__(kScanThreads)
sumset_count_kernel(const unsigned* __restrict__ bitmap, long long nwords, int* __restrict__ sums)
{
    const long long w0 = (long long)blockIdx.x * kWordsPerBlock + threadIdx.x * kWordsPerThread;
    int c = 0;
#pragma unroll
    for (int k = 0; k < kWordsPerThread; ++k)
        if (w0 + k < nwords) c += __popc(bitmap[w0 + k]);
    int total;
    block_exclusive_scan(c, total);
    if (threadIdx.x == 0) sums[blockIdx.x] = total;
}

/* one CTA: block counts -> exclusive block offsets (in place); total -> *nC */
__global__ void __launch_bounds__(kScanThreads)
sumset_scan_kernel(int* __restrict__ sums, long long nblocks, int* __restrict__ nC)
{
    int carry = 0;
    for (long long b0 = 0; b0 < nblocks; b0 += kScanThreads) {
        const long long b = b0 + threadIdx.x;
        const int v = b < nblocks ? sums[b] : 0;
        int total;
        const int ex = block_exclusive_scan(v, total);
        if (b < nblocks) sums[b] = carry + ex;
        carry += total;
    }
    if (threadIdx.x == 0) *nC = carry;
}

__global__ void __launch_bounds__(kScanThreads)
sumset_write_kernel(const unsigned* __restrict__ bitmap, long long nwords,
                    const int* __restrict__ offs, int n, int nC_cap, int* __restrict__ C_off)
{
    const long long w0 = (long long)blockIdx.x * kWordsPerBlock + threadIdx.x * kWordsPerThread;
    unsigned words[kWordsPerThread];
    int c = 0;
#pragma unroll
    for (int k = 0; k < kWordsPerThread; ++k) {
        words[k] = w0 + k < nwords ? bitmap[w0 + k] : 0u;
        c += __popc(words[k]);
    }
    int total;
    int rank = offs[blockIdx.x] + block_exclusive_scan(c, total);
#pragma unroll
    for (int k = 0; k < kWordsPerThread; ++k) {
        unsigned m = words[k];
        while (m) {
            const int bit = __ffs(m) - 1;
            m &= m - 1;
            if (rank < nC_cap) C_off[rank] = (int)((w0 + k) * 32 + bit - (n - 1));
            ++rank;
        }
    }
}

static int sumset(long long n, const int* d_A_off, const int* d_nA, int nA_cap, const int* d_B_off,
                  int nB, int* d_C_off, int* d_nC, int nC_cap, const ChainWork& w,
                  cudaStream_t stream)
{
    DIA_TRY_CUDA(cudaMemsetAsync(w.bitmap, 0, (size_t)w.nwords * 4, stream));
    const long long pairs = (long long)nA_cap * nB;
    if (pairs > 0) {
        const int grid = (int)std::min<long long>((pairs + 255) / 256, 8LL * num_sms());
        sumset_mark_kernel<<<grid, 256, 0, stream>>>(d_A_off, d_nA, nA_cap, d_B_off, nB, (int)n,
                                                     w.bitmap);
        DIA_TRY_CUDA(cudaGetLastError());
    }
    sumset_count_kernel<<<(unsigned)w.nblocks, kScanThreads, 0, stream>>>(w.bitmap, w.nwords,
                                                                          w.block_sums);
    DIA_TRY_CUDA(cudaGetLastError());
    sumset_scan_kernel<<<1, kScanThreads, 0, stream>>>(w.block_sums, w.nblocks, d_nC);
    DIA_TRY_CUDA(cudaGetLastError());
    sumset_write_kernel<<<(unsigned)w.nblocks, kScanThreads, 0, stream>>>(
        w.bitmap, w.nwords, w.block_sums, (int)n, nC_cap, d_C_off);
    DIA_TRY_CUDA(cudaGetLastError());
    return DIA_OK;
}

static int check_args(long long n, int nA_cap, int nB, int nC_cap, int64_t work_bytes,
                      const ChainWork& w, const char* who)
{
    if (n <= 0 || n + kTile >= (1LL << 31) || nA_cap < 0 || nB < 0 || nC_cap < 0)
        return fail(DIA_ERR_INVALID, std::string(who) + ": bad sizes");
    if (work_bytes < (int64_t)w.bytes)
        return fail(DIA_ERR_INVALID, std::string(who) + ": workspace smaller than "
                                                        "dia_spmspm_device_workspace()");
    return DIA_OK;
}

}  // namespace dia

using namespace dia;

extern "C" int64_t dia_spmspm_device_workspace(int64_t n, int nA_cap, int nB, int nC_cap)
{
    (void)nB;
    if (n <= 0 || nA_cap < 0 || nC_cap < 0) return -1;
    return (int64_t)chain_layout(nullptr, n, nA_cap, nC_cap).bytes;
}

extern "C" int dia_spmspm_symbolic_device(int64_t n, const int* d_A_off, const int* d_nA, int nA_cap,
                                          const int* d_B_off, int nB, int* d_C_off, int* d_nC,
                                          int nC_cap, void* d_work, int64_t work_bytes,
                                          cudaStream_t stream)
{
    if (!d_A_off || !d_nA || !d_B_off || !d_C_off || !d_nC || !d_work)
        return fail(DIA_ERR_INVALID, "dia_spmspm_symbolic_device: null pointer");
    const ChainWork w = chain_layout(d_work, n, nA_cap, nC_cap);
    int rc = check_args(n, nA_cap, nB, nC_cap, work_bytes, w, "dia_spmspm_symbolic_device");
    if (rc) return rc;
    return sumset(n, d_A_off, d_nA, nA_cap, d_B_off, nB, d_C_off, d_nC, nC_cap, w, stream);
}

extern "C" int dia_spmspm_rows_device(int64_t n, const int* d_A_off, const int* d_nA, int nA_cap,
                                      const float* d_A_vals, int64_t A_stride, const int* d_B_off,
                                      int nB, const float* d_B_vals, int64_t B_stride,
                                      int* d_C_off, int* d_nC, int nC_cap, float* d_C_vals,
                                      int64_t C_stride, void* d_work, int64_t work_bytes,
                                      cudaStream_t stream)
{
    if (!d_A_off || !d_nA || !d_B_off || !d_C_off || !d_nC || !d_work || !d_A_vals ||
        !d_B_vals || !d_C_vals)
        return fail(DIA_ERR_INVALID, "dia_spmspm_rows_device: null pointer");
    const ChainWork w = chain_layout(d_work, n, nA_cap, nC_cap);
    int rc = check_args(n, nA_cap, nB, nC_cap, work_bytes, w, "dia_spmspm_rows_device");
    if (rc) return rc;
    if (A_stride < n || B_stride < n || C_stride < n)
        return fail(DIA_ERR_INVALID, "dia_spmspm_rows_device: every operand holds all n rows, "
                                     "so each stride must be >= n");
    rc = sumset(n, d_A_off, d_nA, nA_cap, d_B_off, nB, d_C_off, d_nC, nC_cap, w, stream);
    if (rc || nC_cap == 0) return rc;
    rc = build_generic_terms_rows(n, d_A_off, nA_cap, d_B_off, nB, d_C_off, nC_cap, A_stride,
                                  B_stride, 0, 0, n, C_stride, 0, 0, n, w.terms, w.outs, stream,
                                  d_nA, d_nC);
    if (rc) return rc;
    return launch_pair_sum(d_A_vals, d_B_vals, d_C_vals, w.outs, w.terms, nC_cap, 0, (int)n, false,
                           stream, -1.0f, d_nC, 8);
}
