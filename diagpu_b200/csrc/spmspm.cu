/*
 * spmspm.cu -- diagonal-pair SpMSpM numeric phase for sm_100a.
 *
 * C = A*B in diagonal storage: output diagonal dc receives, for every pair
 * (a, b) with da + db = dc, the shifted elementwise product
 *     C[i, i+dc] += A[i, i+da] * B[i+da, i+dc].
 * Two kernels:
 *   pair_plan_kernel  -- one CTA per output diagonal resolves its pairs on the
 *                        device (B found by lookup table or by offset), in A
 *                        storage order, with an order-preserving ballot
 *                        compaction, and writes the term list (element
 *                        offsets + valid rows) to stream-ordered scratch.
 *   pair_sum_kernel   -- persistent CTAs walk (output diagonal, run of row
 *                        tiles) work items, output diagonal fastest, so the A and B
 *                        rows of one tile stay in L2 while all output
 *                        diagonals of that tile are produced.  Each output
 *                        value is accumulated in a register and stored once:
 *                        no atomics, no shared-memory accumulation, and the
 *                        summation order of the reference CPU oracle
 *                        (spmspm/bench_spmspm.cu:392-403).
 * The bound is HBM: bytes 4*(nnzA + nnzB + nnzC) for 2*sum(overlap) flops.
 */
#include <algorithm>

#include "../../include/diagpu_b200.h"
#include "dia_core.cuh"

namespace dia {


/* A diagonal storage scheme reduced to "element offset of row 0" plus the
 * rows where the diagonal holds a stored value. */
struct LayoutDesc {
    int kind;                /* 0 rows layout, 1 HM (size_t starts), 2 HM (int starts) */
    const int* off;          /* device offsets (read for output diagonals) */
    const size_t* st64;
    const int* st32;
    const int* len;
    long long stride;        /* kind 0 */
    long long vrow0;         /* kind 0: global row of element 0 */
    int rlo, rhi;            /* kind 0: rows present in the buffer */
    int n;                   /* matrix order */
};

__device__ __forceinline__ void diag_range(const LayoutDesc& L, int k, int d, long long& base,
                                           int& lo, int& hi)
{
    if (L.kind == 0) {
        base = (long long)k * L.stride - L.vrow0;
        lo = max(max(0, -d), L.rlo);
        hi = min(min(L.n, L.n - d), L.rhi);
    } else {
        const long long s = L.kind == 1 ? (long long)L.st64[k] : (long long)L.st32[k];
        const int m = min(d, 0);
        base = s + m;
        lo = -m;
        hi = L.len[k] - m;
    }
}

struct PlanArgs {
    LayoutDesc A, B, C;
    int nA, nB, nC;
    const int* B_off;     /* used when B_lookup is null */
    const int* B_lookup;  /* [2n-1] or null */
    int row_lo, row_hi;   /* output rows of this call */
    int stride_terms;     /* term slots per output diagonal (>= pairs) */
    Term* terms;
    OutDesc* outs;
    /* optional device-resident counts (a device-side chain step): nA and nC
     * above are then capacities; output diagonals past the device count
     * get an empty descriptor */
    const int* nA_dev;
    const int* nC_dev;
};

constexpr int kBoffSmem = 2048;

__global__ void __launch_bounds__(kBlock) pair_plan_kernel(PlanArgs p)
{
    __shared__ int s_boff[kBoffSmem];
    __shared__ int s_warp[kBlock / 32];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const bool boff_smem = !p.B_lookup && p.nB <= kBoffSmem;
    if (boff_smem)
        for (int b = tid; b < p.nB; b += kBlock) s_boff[b] = p.B_off[b];
    __syncthreads();
    const int n = p.A.n;
    const int nA = p.nA_dev ? min(*p.nA_dev, p.nA) : p.nA;
    const int nC = p.nC_dev ? min(*p.nC_dev, p.nC) : p.nC;

    for (int c = blockIdx.x; c < p.nC; c += gridDim.x) {
        if (c >= nC) {
            if (tid == 0) p.outs[c] = OutDesc{0, 0, 0, 0, 0, c * p.stride_terms, c * p.stride_terms};
            continue;
        }
        const int dc = p.C.off[c];
        OutDesc od;
        int olo, ohi;
        diag_range(p.C, c, dc, od.o, olo, ohi);
        olo = max(olo, p.row_lo);
        ohi = min(ohi, p.row_hi);
        if (p.C.kind == 0) {
            od.wlo = (int)max((long long)p.row_lo, p.C.vrow0);
            od.whi = (int)min((long long)p.row_hi, p.C.vrow0 + p.C.stride);
        } else {
            od.wlo = olo;
            od.whi = ohi;
        }
        if (ohi < olo) ohi = olo;
        od.olo = olo;
        od.ohi = ohi;
        od.t0 = c * p.stride_terms;
        int count = 0;
        for (int a0 = 0; a0 < nA; a0 += kBlock) {
            const int a = a0 + tid;
            bool valid = false;
            Term t;
            if (a < nA && olo < ohi) {
                const int da = p.A.off[a];
                const long long db = (long long)dc - da;
                int b = -1;
                if (p.B_lookup) {
                    if (db > -n && db < n) b = p.B_lookup[db + n - 1];
                } else {
                    for (int bb = 0; bb < p.nB; ++bb) {
                        const int o = boff_smem ? s_boff[bb] : p.B_off[bb];
                        if (o == db) b = bb; /* last match, as the reference's map */
                    }
                }
                if (b >= 0) {
                    long long ua, ub;
                    int alo, ahi, blo, bhi;
                    diag_range(p.A, a, da, ua, alo, ahi);
                    diag_range(p.B, b, (int)db, ub, blo, bhi);
                    t.u = ua;
                    t.v = ub + da;
                    t.lo = max(max(alo, blo - da), olo);
                    t.hi = min(min(ahi, bhi - da), ohi);
                    valid = t.lo < t.hi;
                }
            }
            const unsigned m = __ballot_sync(0xffffffffu, valid);
            if (lane == 0) s_warp[warp] = __popc(m);
            __syncthreads();
            int woff = 0, total = 0;
            for (int w = 0; w < kBlock / 32; ++w) {
                woff += w < warp ? s_warp[w] : 0;
                total += s_warp[w];
            }
            if (valid) {
                const int pos = count + woff + __popc(m & ((1u << lane) - 1u));
                p.terms[od.t0 + pos] = t;
            }
            count += total;
            __syncthreads();
        }
        od.t1 = od.t0 + count;
        if (tid == 0) p.outs[c] = od;
    }
}

struct SumArgs {
    const float* U;
    const float* V;
    float* O;
    const OutDesc* outs;
    const Term* terms;
    int nOut;
    int row_lo;
    int row_hi;
    int ntiles;
    int tiles_per_item;  /* consecutive row tiles one work item covers; 0: chosen
                          * on the device from the term counts in outs */
    const int* nOut_dev; /* optional device-resident count; nOut is then a capacity */
};

/* Persistent CTAs walk work items (output diagonal c, run of tiles), c
 * fastest.  An item loads its term list into shared memory once and then
 * sweeps its tiles, so the descriptor/term fetch latency is paid once per
 * tiles_per_item tiles. */
template <bool ACCUM, int ILP, int BATCH>
__global__ void __launch_bounds__(kBlock) pair_sum_kernel(SumArgs s)
{
    constexpr int kTile = kBlock * ILP;
    __shared__ Term s_t[kMaxTerms];
    const int nOut = s.nOut_dev ? min(*s.nOut_dev, s.nOut) : s.nOut;
    if (s.tiles_per_item == 0) {
        /* the host could not see the plan: every CTA sums the term counts
         * (a few thousand descriptors at most, L2-resident) and applies the
         * host rule of launch_pair_sum_t */
        __shared__ long long s_terms;
        if (threadIdx.x == 0) s_terms = 0;
        __syncthreads();
        long long mine = 0;
        for (int c = threadIdx.x; c < nOut; c += kBlock) mine += s.outs[c].t1 - s.outs[c].t0;
        atomicAdd((unsigned long long*)&s_terms, (unsigned long long)mine);
        __syncthreads();
        const long long tiles = (long long)nOut * s.ntiles;
        int tpi = 1;
        if (s_terms <= 2LL * nOut)
            tpi = (int)max(1LL, min(16LL, tiles / (8LL * gridDim.x)));
        s.tiles_per_item = tpi;
    }
    const int nchunks = (s.ntiles + s.tiles_per_item - 1) / s.tiles_per_item;
    const long long items = (long long)nOut * nchunks;
    for (long long it = blockIdx.x; it < items; it += gridDim.x) {
        const int c = (int)(it % nOut);
        const int tfirst = (int)(it / nOut) * s.tiles_per_item;
        const int tlast = min(s.ntiles, tfirst + s.tiles_per_item);
        const OutDesc od = s.outs[c];
        const int span_lo = s.row_lo + tfirst * kTile, span_hi = s.row_lo + tlast * kTile;
        if (max(od.wlo, span_lo) >= min(od.whi, span_hi)) continue;
        const int nt = od.t1 - od.t0;
        const bool resident = nt <= kMaxTerms;
        if (resident) {
            __syncthreads();
            for (int q = threadIdx.x; q < nt; q += kBlock) s_t[q] = s.terms[od.t0 + q];
            __syncthreads();
        }
        for (int tile = tfirst; tile < tlast; ++tile) {
            const int tile_lo = s.row_lo + tile * kTile;
            const int wlo = max(od.wlo, tile_lo);
            const int whi = min(min(od.whi, tile_lo + kTile), s.row_hi);
            if (wlo >= whi) continue;
            const int r0 = tile_lo + (int)threadIdx.x;
            float acc[ILP];
#pragma unroll
            for (int j = 0; j < ILP; ++j) acc[j] = 0.0f;
            if (resident) {
                accumulate_terms<false, ILP, BATCH>(s.U, s.V, s_t, nt, tile_lo, r0, acc);
            } else {
                for (int t0 = od.t0; t0 < od.t1; t0 += kMaxTerms) {
                    const int m = min(kMaxTerms, od.t1 - t0);
                    __syncthreads();
                    for (int q = threadIdx.x; q < m; q += kBlock) s_t[q] = s.terms[t0 + q];
                    __syncthreads();
                    accumulate_terms<false, ILP, BATCH>(s.U, s.V, s_t, m, tile_lo, r0, acc);
                }
            }
#pragma unroll
            for (int j = 0; j < ILP; ++j) {
                const int i = r0 + j * kBlock;
                if (i >= wlo && i < whi) {
                    const float v = (i >= od.olo && i < od.ohi) ? acc[j] : 0.0f;
                    float* dst = s.O + od.o + i;
                    if (ACCUM)
                        *dst = __fadd_rn(*dst, v);
                    else
                        __stcs(dst, v);
                }
            }
        }
    }
}

/* Launch the persistent pair-sum kernel over nOut output diagonals and the
 * rows [row_lo, row_hi). */
template <int ILP, int BATCH>
static int launch_pair_sum_t(const float* U, const float* V, float* O, const OutDesc* outs,
                             const Term* terms, int nOut, int row_lo, int row_hi,
                             bool accumulate, float avg_terms, cudaStream_t stream,
                             const int* nOut_dev)
{
    constexpr int kTile = kBlock * ILP;
    SumArgs s{U, V, O, outs, terms, nOut, row_lo, row_hi, (row_hi - row_lo + kTile - 1) / kTile, 1,
              nOut_dev};
    const void* k = accumulate ? (const void*)pair_sum_kernel<true, ILP, BATCH>
                               : (const void*)pair_sum_kernel<false, ILP, BATCH>;
    const long long slots = persistent_blocks(k, 0);
    const long long tiles = (long long)nOut * s.ntiles;
    /* Long runs of tiles per item amortise the item set-up, which pays off
     * when output diagonals have few terms; with many terms the items of
     * one run progress at very different rates and evict each other's B
     * rows from L2 (measured: 11x the algorithmic DRAM reads on a 27-point
     * stencil product at 16 tiles per item, 1.2x at one). */
    s.tiles_per_item = 1;
    if (avg_terms >= 0.0f && avg_terms <= 2.0f)
        s.tiles_per_item = (int)std::max(1LL, std::min(16LL, tiles / (8 * slots)));
    long long grid;
    if (avg_terms < 0.0f && nOut_dev == nullptr) {
        /* term counts unknown on the host (device-planned products) */
        s.tiles_per_item = 0;
        grid = std::min(slots, tiles);
    } else {
        const int nchunks = (s.ntiles + s.tiles_per_item - 1) / s.tiles_per_item;
        grid = std::min(slots, (long long)nOut * nchunks);
    }
    if (accumulate)
        pair_sum_kernel<true, ILP, BATCH><<<(unsigned)grid, kBlock, 0, stream>>>(s);
    else
        pair_sum_kernel<false, ILP, BATCH><<<(unsigned)grid, kBlock, 0, stream>>>(s);
    DIA_TRY_CUDA(cudaGetLastError());
    return DIA_OK;
}

/* Launch the persistent pair-sum kernel over nOut output diagonals and the
 * rows [row_lo, row_hi). */
int launch_pair_sum(const float* U, const float* V, float* O, const OutDesc* outs,
                    const Term* terms, int nOut, int row_lo, int row_hi, bool accumulate,
                    cudaStream_t stream, float avg_terms, const int* nOut_dev,
                    int rows_per_thread)
{
    if (nOut <= 0 || row_hi <= row_lo) return DIA_OK;
    if (rows_per_thread == 8)
        return launch_pair_sum_t<8, 4>(U, V, O, outs, terms, nOut, row_lo, row_hi, accumulate,
                                       avg_terms, stream, nOut_dev);
    return launch_pair_sum_t<4, 4>(U, V, O, outs, terms, nOut, row_lo, row_hi, accumulate,
                                   avg_terms, stream, nOut_dev);
}

static int run_planned(PlanArgs p, const float* U, const float* V, float* O,
                       cudaStream_t stream)
{
    if (p.nC <= 0 || p.row_hi <= p.row_lo) return DIA_OK;
    p.stride_terms = std::max(p.nA, 1);
    const size_t term_bytes = (size_t)p.nC * p.stride_terms * sizeof(Term);
    const size_t out_bytes = (size_t)p.nC * sizeof(OutDesc);
    void* ws = nullptr;
    DIA_TRY_CUDA(cudaMallocAsync(&ws, term_bytes + out_bytes, stream));
    p.terms = (Term*)ws;
    p.outs = (OutDesc*)((char*)ws + term_bytes);
    const int grid = std::min(p.nC, 8 * num_sms());
    pair_plan_kernel<<<grid, kBlock, 0, stream>>>(p);
    cudaError_t e = cudaGetLastError();
    int rc = e == cudaSuccess ? DIA_OK : cuda_fail(e, "pair_plan_kernel launch");
    if (rc == DIA_OK)
        rc = launch_pair_sum(U, V, O, p.outs, p.terms, p.nC, p.row_lo, p.row_hi, false, stream);
    cudaError_t ef = cudaFreeAsync(ws, stream);
    if (rc == DIA_OK && ef != cudaSuccess) rc = cuda_fail(ef, "cudaFreeAsync");
    return rc;
}

/* Term lists of a rows-layout product written into caller buffers
 * (terms: nC * nA slots, outs: nC), for plans that keep them. */
int build_generic_terms_rows(long long n, const int* d_A_off, int nA, const int* d_B_off, int nB,
                             const int* d_C_off, int nC, long long A_stride,
                             long long B_stride, long long b_vrow0, long long b_lo,
                             long long b_hi, long long C_stride, long long vrow0,
                             long long row_lo, long long row_hi, Term* terms, OutDesc* outs,
                             cudaStream_t stream, const int* nA_dev, const int* nC_dev)
{
    const int in = (int)n;
    PlanArgs p{};
    p.nA_dev = nA_dev;
    p.nC_dev = nC_dev;
    p.A = LayoutDesc{0, d_A_off, nullptr, nullptr, nullptr, A_stride, vrow0, (int)vrow0,
                     (int)std::min<long long>(vrow0 + A_stride, n), in};
    p.B = LayoutDesc{0, d_B_off, nullptr, nullptr, nullptr, B_stride, b_vrow0,
                     (int)std::max<long long>(b_lo, 0), (int)std::min<long long>(b_hi, n), in};
    p.C = LayoutDesc{0, d_C_off, nullptr, nullptr, nullptr, C_stride, vrow0, (int)vrow0,
                     (int)std::min<long long>(vrow0 + C_stride, n), in};
    p.nA = nA;
    p.nB = nB;
    p.nC = nC;
    p.B_off = d_B_off;
    p.row_lo = (int)row_lo;
    p.row_hi = (int)row_hi;
    p.stride_terms = std::max(nA, 1);
    p.terms = terms;
    p.outs = outs;
    pair_plan_kernel<<<std::min(nC, 8 * num_sms()), kBlock, 0, stream>>>(p);
    DIA_TRY_CUDA(cudaGetLastError());
    return DIA_OK;
}

}  // namespace dia

using namespace dia;

extern "C" int dia_spmspm_hm(const float* d_A_values, const size_t* d_A_starts, const int* d_A_off,
                             const int* d_A_len, int A_ndiag, const float* d_B_values,
                             const size_t* d_B_starts, const int* d_B_len, const int* d_B_lookup,
                             float* d_C_values, const size_t* d_C_starts, const int* d_C_off,
                             const int* d_C_len, int C_ndiag, int n, cudaStream_t stream)
{
    if (n < 0 || A_ndiag < 0 || C_ndiag < 0)
        return fail(DIA_ERR_INVALID, "dia_spmspm_hm: negative size");
    if (n == 0 || C_ndiag == 0) return DIA_OK;
    if (!d_C_values || !d_C_starts || !d_C_off || !d_C_len ||
        (A_ndiag > 0 && (!d_A_values || !d_A_starts || !d_A_off || !d_A_len || !d_B_values ||
                         !d_B_starts || !d_B_len || !d_B_lookup)))
        return fail(DIA_ERR_INVALID, "dia_spmspm_hm: null pointer");
    if ((long long)n + kTile >= (1LL << 31))
        return fail(DIA_ERR_UNSUPPORTED, "dia_spmspm_hm: n beyond int32 range");
    PlanArgs p{};
    p.A = LayoutDesc{1, d_A_off, d_A_starts, nullptr, d_A_len, 0, 0, 0, 0, n};
    p.B = LayoutDesc{1, nullptr, d_B_starts, nullptr, d_B_len, 0, 0, 0, 0, n};
    p.C = LayoutDesc{1, d_C_off, d_C_starts, nullptr, d_C_len, 0, 0, 0, 0, n};
    p.nA = A_ndiag;
    p.nB = 0;
    p.nC = C_ndiag;
    p.B_lookup = d_B_lookup;
    p.row_lo = 0;
    p.row_hi = n;
    return run_planned(p, d_A_values, d_B_values, d_C_values, stream);
}

extern "C" int dia_spmspm_rows(int64_t n, const float* d_A_vals, int64_t A_stride,
                               const int* d_A_off, int nA, const float* d_B_vals,
                               int64_t B_stride, int64_t b_vrow0, int64_t b_lo, int64_t b_hi,
                               const int* d_B_off, int nB, float* d_C_vals, int64_t C_stride,
                               const int* d_C_off, int nC, int64_t vrow0, int64_t row_lo,
                               int64_t row_hi, cudaStream_t stream)
{
    if (n < 0 || nA < 0 || nB < 0 || nC < 0 || A_stride < 0 || B_stride < 0 || C_stride < 0)
        return fail(DIA_ERR_INVALID, "dia_spmspm_rows: negative size");
    if (n + kTile >= (1LL << 31))
        return fail(DIA_ERR_UNSUPPORTED, "dia_spmspm_rows: n beyond int32 range");
    row_lo = std::max<int64_t>(row_lo, vrow0);
    row_hi = std::min<int64_t>(row_hi, vrow0 + C_stride);
    if (nC == 0 || row_hi <= row_lo) return DIA_OK;
    if (!d_C_vals || !d_C_off || (nA > 0 && (!d_A_vals || !d_A_off || !d_B_vals || !d_B_off)))
        return fail(DIA_ERR_INVALID, "dia_spmspm_rows: null pointer");
    if (b_lo < b_vrow0 || b_hi > b_vrow0 + B_stride)
        return fail(DIA_ERR_INVALID, "dia_spmspm_rows: B rows outside the B buffer");
    const int in = (int)n;
    PlanArgs p{};
    p.A = LayoutDesc{0, d_A_off, nullptr, nullptr, nullptr, A_stride, vrow0, (int)vrow0,
                     (int)std::min<int64_t>(vrow0 + A_stride, n), in};
    p.B = LayoutDesc{0, d_B_off, nullptr, nullptr, nullptr, B_stride, b_vrow0,
                     (int)std::max<int64_t>(b_lo, 0), (int)std::min<int64_t>(b_hi, n), in};
    p.C = LayoutDesc{0, d_C_off, nullptr, nullptr, nullptr, C_stride, vrow0, (int)vrow0,
                     (int)std::min<int64_t>(vrow0 + C_stride, n), in};
    p.nA = nA;
    p.nB = nB;
    p.nC = nC;
    p.B_off = d_B_off;
    p.B_lookup = nullptr;
    p.row_lo = (int)row_lo;
    p.row_hi = (int)row_hi;
    return run_planned(p, d_A_vals, d_B_vals, d_C_vals, stream);
}

/* ------------------------------------------------------------------------
 * Allocation-free variant of dia_spmspm_hm.
 *
 * dia_spmspm_hm takes its pair-plan scratch from the stream-ordered
 * allocator.  Some callers cannot allocate device memory at call time: an
 * application whose own allocator has reserved all device memory up front,
 * a solver loop that runs under a fixed memory budget, or code that must not
 * touch the driver's allocator while it runs.  This entry point keeps the
 * plan in a file-scope device array instead, so it performs no allocation of
 * any kind.  Its limit is the size of that array.
 * ------------------------------------------------------------------------ */
#include <mutex>

namespace dia {

/* 8 MiB of plan: C_ndiag * A_ndiag * 24 + C_ndiag * 32 bytes must fit. */
constexpr size_t kStaticPlanBytes = size_t(8) << 20;
static __device__ __align__(256) unsigned char g_static_plan[kStaticPlanBytes];

/* Device address of g_static_plan on the current device, looked up once per
 * device (the host-side symbol is only a stand-in, never a device pointer). */
static int static_plan_address(void** out)
{
    constexpr int kMaxDevices = 64;
    static std::mutex mu;
    static void* addr[kMaxDevices] = {};
    int dev = 0;
    DIA_TRY_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kMaxDevices)
        return fail(DIA_ERR_UNSUPPORTED, "dia_spmspm_hm_noalloc: device index above 63");
    std::lock_guard<std::mutex> g(mu);
    if (!addr[dev]) {
        void* p = nullptr;
        DIA_TRY_CUDA(cudaGetSymbolAddress(&p, g_static_plan));
        addr[dev] = p;
    }
    *out = addr[dev];
    return DIA_OK;
}

}  // namespace dia

extern "C" int dia_spmspm_hm_noalloc(const float* d_A_values, const size_t* d_A_starts,
                                     const int* d_A_off, const int* d_A_len, int A_ndiag,
                                     const float* d_B_values, const size_t* d_B_starts,
                                     const int* d_B_len, const int* d_B_lookup,
                                     float* d_C_values, const size_t* d_C_starts,
                                     const int* d_C_off, const int* d_C_len, int C_ndiag, int n,
                                     cudaStream_t stream)
{
    if (n < 0 || A_ndiag < 0 || C_ndiag < 0)
        return fail(DIA_ERR_INVALID, "dia_spmspm_hm_noalloc: negative size");
    if (n == 0 || C_ndiag == 0) return DIA_OK;
    if (!d_C_values || !d_C_starts || !d_C_off || !d_C_len ||
        (A_ndiag > 0 && (!d_A_values || !d_A_starts || !d_A_off || !d_A_len || !d_B_values ||
                         !d_B_starts || !d_B_len || !d_B_lookup)))
        return fail(DIA_ERR_INVALID, "dia_spmspm_hm_noalloc: null pointer");
    if ((long long)n + kTile >= (1LL << 31))
        return fail(DIA_ERR_UNSUPPORTED, "dia_spmspm_hm_noalloc: n beyond int32 range");
    const int stride_terms = std::max(A_ndiag, 1);
    const size_t term_bytes = (size_t)C_ndiag * stride_terms * sizeof(Term);
    const size_t need = term_bytes + (size_t)C_ndiag * sizeof(OutDesc);
    if (need > kStaticPlanBytes)
        return fail(DIA_ERR_CAPACITY,
                    "dia_spmspm_hm_noalloc: plan needs " + std::to_string(need) +
                        " bytes (C_ndiag * A_ndiag * 24 + C_ndiag * 32) but the static buffer "
                        "holds " + std::to_string(kStaticPlanBytes) + "; use dia_spmspm_hm");
    void* ws = nullptr;
    const int rc = static_plan_address(&ws);
    if (rc != DIA_OK) return rc;
    PlanArgs p{};
    p.A = LayoutDesc{1, d_A_off, d_A_starts, nullptr, d_A_len, 0, 0, 0, 0, n};
    p.B = LayoutDesc{1, nullptr, d_B_starts, nullptr, d_B_len, 0, 0, 0, 0, n};
    p.C = LayoutDesc{1, d_C_off, d_C_starts, nullptr, d_C_len, 0, 0, 0, 0, n};
    p.nA = A_ndiag;
    p.nB = 0;
    p.nC = C_ndiag;
    p.B_lookup = d_B_lookup;
    p.row_lo = 0;
    p.row_hi = n;
    p.stride_terms = stride_terms;
    /* every descriptor and every term the sum kernel reads is rewritten by
     * the plan kernel first, so nothing left by an earlier call is used */
    p.terms = (Term*)ws;
    p.outs = (OutDesc*)((char*)ws + term_bytes);
    pair_plan_kernel<<<std::min(C_ndiag, 8 * num_sms()), kBlock, 0, stream>>>(p);
    DIA_TRY_CUDA(cudaGetLastError());
    return launch_pair_sum(d_A_values, d_B_values, d_C_values, p.outs, p.terms, C_ndiag, 0, n,
                           false, stream);
}
