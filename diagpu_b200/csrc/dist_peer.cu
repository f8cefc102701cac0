/*
 * dist_peer.cu -- row-partitioned SpMV with the x halo moved by the kernel
 * itself over NVLink (peer stores), one launch per step.
 *
 * Rank r owns rows [r0, r1) and the matching x columns.  Row i needs the x
 * columns i + d for every offset d, so the rows within max|d| of a block edge
 * need a neighbour's columns (the halo).  Instead of an NCCL send/receive
 * followed by separate boundary launches, one kernel does the whole step:
 *
 *   - its first CTAs copy this rank's edge columns straight into the
 *     neighbours' receive buffers (plain stores through CUDA IPC mappings of
 *     the neighbours' memory), then the last of them publishes the step
 *     number in the neighbour's flag word (system-scope release);
 *   - the interior tiles (all columns local) never wait;
 *   - the boundary tiles are dispatched a quarter of the way through the
 *     grid; one thread of each spins on the flag (system-scope acquire) with
 *     a time limit, so by the time they run the neighbour's columns have
 *     normally arrived long ago and the wait costs nothing.  On time-out the
 *     kernel sets DIA_DIST_TIMEOUT in the status word and finishes without
 *     waiting.
 *
 * Receive buffers are double-buffered by step parity.  Step s writes buffer
 * s & 1; a neighbour can only write that buffer again at step s + 2, which it
 * reaches after waiting for this rank's step s + 1 flag, published when this
 * rank's step s kernel has finished (stream order).  Every rank therefore
 * waits for every existing neighbour's flag each step, even when its offsets
 * need no columns from that side.
 *
 * The summation is the single-GPU kernel's: each diagonal's term is split
 * into up to three row segments (columns from the left halo, the own block,
 * the right halo) that cover disjoint rows, so every row still adds its
 * terms in offset storage order and the result equals the whole-matrix SpMV
 * bit for bit.  The reference has no multi-GPU path.
 */
#include "../../include/diagpu_b200.h"
#include "dia_core.cuh"

namespace dia {

constexpr int kPushCtas = 4;      /* CTAs per side that copy the halo */
constexpr int kPeerMaxDiags = 128; /* 3 segments per diagonal fit kMaxTerms */

__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long* p)
{
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void st_release_sys(unsigned long long* p, unsigned long long v)
{
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ unsigned long long global_ns()
{
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

struct PeerSpmvArgs {
    const float* vals;
    const float* x_own;   /* columns [r0, r1) */
    float* y;             /* row i at y[i - vrow0] */
    const int* off;
    int K;
    int r0, r1;           /* rows computed = own columns */
    int xlo, xhi;         /* halo window [xlo, r0) and [r1, xhi) */
    int ncols;
    long long vrow0, stride;
    int ntiles, nlow, nhigh;
    unsigned long long step;
    DiaPeerHalo h;
};

/* Thread 0 waits (bounded) until *flag >= step. */
__device__ __forceinline__ void wait_flag(const unsigned long long* flag, unsigned long long step,
                                          long long timeout_ns, unsigned int* status)
{
    if (threadIdx.x != 0 || flag == nullptr) return;
    if (ld_acquire_sys(flag) >= step) return;
    const unsigned long long t0 = global_ns();
    while (ld_acquire_sys(flag) < step) {
        if ((long long)(global_ns() - t0) > timeout_ns) {
            atomicOr(status, (unsigned)DIA_DIST_TIMEOUT);
            return;
        }
        __nanosleep(128);
    }
}

__global__ void __launch_bounds__(kBlock, 8) peer_spmv_kernel(PeerSpmvArgs a)
{
    __shared__ Term s_t[kMaxTerms];
    __shared__ int s_nt;
    const int b = (int)blockIdx.x;
    const int par = (int)(a.step & 1ull);

    /* 1. push this rank's edge columns to the neighbours */
    const int npush = (a.h.has_left + a.h.has_right) * kPushCtas;
    if (b < npush) {
        const int side = (a.h.has_left && b < kPushCtas) ? 0 : 1;
        const int j = b % kPushCtas;
        long long lo, hi;
        float* dst;
        unsigned long long* flag;
        if (side == 0) {
            lo = a.r0;
            hi = a.h.send_left_hi;
            dst = a.h.peer_left_halo_hi[par] - a.r0;
            flag = a.h.peer_left_flag_hi;
        } else {
            lo = a.h.send_right_lo;
            hi = a.r1;
            dst = a.h.peer_right_halo_lo[par] - a.h.send_right_lo;
            flag = a.h.peer_right_flag_lo;
        }
        const float* src = a.x_own - a.r0;
        for (long long c = lo + (long long)j * kBlock + threadIdx.x; c < hi;
             c += (long long)kPushCtas * kBlock)
            dst[c] = src[c];
        __threadfence_system();
        __syncthreads();
        if (threadIdx.x == 0) {
            const unsigned long long done = atomicAdd(&a.h.push_count[side], 1ull) + 1ull;
            if (done == a.step * kPushCtas) {
                __threadfence_system();
                st_release_sys(flag, a.step);
            }
        }
    }

    /* 2. which tile: the boundary tiles are dispatched a quarter of the way
     * through the grid.  By then the neighbours' pushes (issued at their
     * kernels' start) have long arrived, and the slower boundary tiles
     * (split terms) are absorbed by the interior tiles that follow instead
     * of forming the kernel's tail. */
    const int interior = a.ntiles - a.nlow - a.nhigh;
    const int nb = a.nlow + a.nhigh;
    const int first = interior / 4;
    int t;
    const bool boundary = b >= first && b < first + nb;
    if (!boundary) {
        t = a.nlow + (b < first ? b : b - nb);
    } else {
        const int q = b - first;
        t = q < a.nlow ? q : a.ntiles - a.nhigh + (q - a.nlow);
    }
    const int tile_lo = a.r0 + t * kTile;
    const int tile_hi = min(tile_lo + kTile, a.r1);

    /* 3. term list: the own-column segment of every diagonal, plus the halo
     * segments that meet this tile (boundary tiles only) */
    if (!boundary) {
        /* every column of an interior tile is this rank's own */
        for (int k = threadIdx.x; k < a.K; k += kBlock) {
            const long long d = a.off[k];
            const long long own_hi = a.r1 < a.ncols ? a.r1 : a.ncols;
            long long lo = a.r0 - d, hi = own_hi - d;
            lo = lo < a.r0 ? a.r0 : lo;
            hi = hi > a.r1 ? a.r1 : hi;
            if (hi < lo) hi = lo;
            Term t;
            t.u = (long long)k * a.stride - a.vrow0;
            t.v = d - a.r0;
            t.lo = (int)lo;
            t.hi = (int)hi;
            s_t[k] = t;
        }
        if (threadIdx.x == 0) s_nt = a.K;
    } else if (threadIdx.x < 32) {
        const int lane = threadIdx.x;
        int base = 0;
        for (int k0 = 0; k0 < a.K; k0 += 32) {
            const int k = k0 + lane;
            /* rows whose column i + d lies in source s (0: left halo,
             * 1: own block, 2: right halo), clipped to the block's rows */
            const long long d = k < a.K ? a.off[k] : 0;
            auto rows_of = [&](int s, long long& lo, long long& hi) {
                const long long own_hi = a.r1 < a.ncols ? a.r1 : a.ncols;
                const long long xhi = a.xhi < a.ncols ? a.xhi : a.ncols;
                const long long c0 = s == 0 ? a.xlo : (s == 1 ? a.r0 : a.r1);
                const long long c1 = s == 0 ? a.r0 : (s == 1 ? own_hi : xhi);
                lo = c0 - d;
                hi = c1 - d;
                lo = lo < a.r0 ? a.r0 : lo;
                hi = hi > a.r1 ? a.r1 : hi;
                return k < a.K && hi > lo && lo < tile_hi && hi > tile_lo;
            };
            unsigned okm = 0;
#pragma unroll
            for (int s = 0; s < 3; ++s) {
                long long lo, hi;
                okm |= rows_of(s, lo, hi) ? 1u << s : 0u;
            }
            const int cnt = __popc(okm);
            /* exclusive prefix of the per-lane counts keeps diagonal order */
            int pre = cnt;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int v = __shfl_up_sync(0xffffffffu, pre, o);
                if (lane >= o) pre += v;
            }
            const int tot = __shfl_sync(0xffffffffu, pre, 31);
            int pos = base + pre - cnt;
#pragma unroll
            for (int s = 0; s < 3; ++s) {
                if (!(okm >> s & 1u)) continue;
                long long lo, hi;
                rows_of(s, lo, hi);
                /* V offsets relative to x_own, in elements; the halo
                 * buffers are other allocations, reached through the flat
                 * address space */
                long long vb;
                if (s == 1)
                    vb = -(long long)a.r0;
                else if (s == 0)
                    vb = (long long)(a.h.halo_lo[par] - a.x_own) - a.xlo;
                else
                    vb = (long long)(a.h.halo_hi[par] - a.x_own) - a.r1;
                Term t;
                t.u = (long long)k * a.stride - a.vrow0;
                t.v = vb + d;
                t.lo = (int)lo;
                t.hi = (int)hi;
                s_t[pos++] = t;
            }
            base += tot;
        }
        if (lane == 0) s_nt = base;
    }

    /* 4. boundary tiles (and the last block, for the step ordering) wait for
     * the neighbours' columns of this step */
    const bool need_lo = a.h.has_left && tile_lo < a.r0 + (a.r0 - a.xlo);
    const bool need_hi = a.h.has_right && tile_hi > a.r1 - (a.xhi - a.r1);
    const bool last = b == (int)gridDim.x - 1;
    if (need_lo || (last && a.h.has_left))
        wait_flag(a.h.flag_lo, a.step, a.h.timeout_ns, a.h.status);
    if (need_hi || (last && a.h.has_right))
        wait_flag(a.h.flag_hi, a.step, a.h.timeout_ns, a.h.status);
    __syncthreads();

    float acc[kILP];
#pragma unroll
    for (int j = 0; j < kILP; ++j) acc[j] = 0.0f;
    const int r0 = tile_lo + (int)threadIdx.x;
    accumulate_terms<true>(a.vals, a.x_own, s_t, s_nt, tile_lo, r0, acc);
#pragma unroll
    for (int j = 0; j < kILP; ++j) {
        const int i = r0 + j * kBlock;
        if (i < a.r1) a.y[i - a.vrow0] = acc[j];
    }
}

}  // namespace dia

using namespace dia;

extern "C" int dia_spmv_rows_peer(const DiaPeerHalo* h, uint64_t step, int64_t n_rows,
                                  int64_t n_cols, int num_diags, const int* d_offsets,
                                  const float* d_vals, int64_t stride, int64_t vrow0, int64_t r0,
                                  int64_t r1, int64_t x_lo, int64_t x_hi, int dmin, int dmax,
                                  const float* d_x_own, float* d_y, cudaStream_t stream)
{
    if (!h || !d_x_own || !d_y || (num_diags > 0 && (!d_offsets || !d_vals)))
        return fail(DIA_ERR_INVALID, "dia_spmv_rows_peer: null pointer");
    if (num_diags < 0 || num_diags > kPeerMaxDiags)
        return fail(DIA_ERR_UNSUPPORTED, "dia_spmv_rows_peer: more than 128 diagonals");
    if (step == 0) return fail(DIA_ERR_INVALID, "dia_spmv_rows_peer: steps count from 1");
    if (r0 < 0 || r1 > n_rows || r1 < r0 || r0 < vrow0 || r1 > vrow0 + stride ||
        x_lo > r0 || x_hi < r1 || x_lo < 0 || x_hi > n_cols)
        return fail(DIA_ERR_INVALID, "dia_spmv_rows_peer: inconsistent block or halo window");
    if (n_rows + kTile >= (1LL << 31) || n_cols >= (1LL << 31))
        return fail(DIA_ERR_UNSUPPORTED, "dia_spmv_rows_peer: dimensions beyond int32 range");
    if ((h->has_left && (!h->flag_lo || !h->peer_left_flag_hi || !h->peer_left_halo_hi[0] ||
                         !h->peer_left_halo_hi[1] || (x_lo < r0 && (!h->halo_lo[0] ||
                                                                     !h->halo_lo[1])))) ||
        (h->has_right && (!h->flag_hi || !h->peer_right_flag_lo || !h->peer_right_halo_lo[0] ||
                          !h->peer_right_halo_lo[1] || (x_hi > r1 && (!h->halo_hi[0] ||
                                                                       !h->halo_hi[1])))) ||
        ((h->has_left || h->has_right) && (!h->push_count || !h->status)))
        return fail(DIA_ERR_INVALID, "dia_spmv_rows_peer: missing peer buffers");
    if ((!h->has_left && x_lo < r0) || (!h->has_right && x_hi > r1))
        return fail(DIA_ERR_INVALID, "dia_spmv_rows_peer: halo columns without a neighbour");
    const long long rows = r1 - r0;
    if (rows == 0) return DIA_OK;
    PeerSpmvArgs a{};
    a.vals = d_vals;
    a.x_own = d_x_own;
    a.y = d_y;
    a.off = d_offsets;
    a.K = num_diags;
    a.r0 = (int)r0;
    a.r1 = (int)r1;
    a.xlo = (int)x_lo;
    a.xhi = (int)x_hi;
    a.ncols = (int)n_cols;
    a.vrow0 = vrow0;
    a.stride = stride;
    a.step = step;
    a.h = *h;
    a.ntiles = (int)((rows + kTile - 1) / kTile);
    /* tiles that read a halo column: tile_lo + dmin < r0, tile_hi - 1 + dmax >= r1 */
    const long long need_lo = h->has_left && dmin < 0 ? -(long long)dmin : 0;
    const long long need_hi = h->has_right && dmax > 0 ? (long long)dmax : 0;
    long long nlow = (need_lo + kTile - 1) / kTile;
    if (nlow > a.ntiles) nlow = a.ntiles;
    long long nhigh = 0;
    if (need_hi > 0) {
        /* the last tile is partial: count tiles whose end exceeds r1 - dmax */
        const long long first = (rows - need_hi) <= 0 ? 0 : (rows - need_hi) / kTile;
        nhigh = a.ntiles - first;
    }
    if (nlow + nhigh > a.ntiles) nhigh = a.ntiles - nlow;
    a.nlow = (int)nlow;
    a.nhigh = (int)nhigh;
    const int npush = (h->has_left + h->has_right) * kPushCtas;
    const int grid = a.ntiles > npush ? a.ntiles : npush;
    if (grid > a.ntiles) {
        /* fewer tiles than pushing CTAs: not a shape this path is for */
        return fail(DIA_ERR_UNSUPPORTED, "dia_spmv_rows_peer: block smaller than 8 tiles");
    }
    peer_spmv_kernel<<<grid, kBlock, 0, stream>>>(a);
    DIA_TRY_CUDA(cudaGetLastError());
    return DIA_OK;
}
