/*
 * spmspm_tiled.cu -- planned, shared-memory-tiled SpMSpM for sm_100a.
 *
 * The generic pair-sum kernel (spmspm.cu) fetches both operands of every
 * product from L2.  For products whose A offsets come in tight groups
 * (stencils, bands) the same B values serve many products, so this path
 * stages them once per row tile:
 *   - a plan (built once on the host, like the reference's host Schedule,
 *     spmspm/bench_spmspm.cu:137-243) groups A's offsets into clusters of
 *     span <= kClusterSpan, and for every (B diagonal, A cluster) pair that
 *     occurs it lays out one shared-memory window holding the B rows that
 *     tile's products touch; A's diagonals get one T-row slot each;
 *   - tile_sum_kernel: persistent CTAs take T-row tiles of the interior rows
 *     (rows whose every term is in range), copy the A slots and the B
 *     windows with 16-byte cp.async, then each warp produces whole output
 *     diagonals for the tile: lanes are rows, every product reads two
 *     conflict-free shared-memory words, and the terms are applied in the
 *     pair order of the reference CPU oracle (spmspm/bench_spmspm.cu:392-403)
 *     with separately rounded multiply and add -- results are bit-identical
 *     to the generic path;
 *   - the few edge rows run through the generic kernel with term lists the
 *     plan also precomputes, so execution needs no scratch allocation.
 */
#include <algorithm>
#include <climits>
#include <map>
#include <vector>

#include "../../include/diagpu_b200.h"
#include "dia_core.cuh"

namespace dia {

struct RunBlock;
struct RunPairDesc;
struct RunPairPlan {
    int P = 0, Q = 0, nblk = 0, i_lo = 0, i_hi = 0;
    RunBlock* d_blks = nullptr;
    RunPairDesc* d_rps = nullptr;
};
bool runpair_plan_build(const int* hA, int nA, const int* hB, int nB, const int* hC, int nC,
                        long long A_stride, long long B_stride, long long C_stride,
                        long long vrow0, long long b_vrow0, int b_lo, int b_hi, int rows_lo,
                        int rows_hi, RunPairPlan* rp);
void runpair_plan_free(RunPairPlan* rp);
int runpair_launch(const RunPairPlan* rp, const float* A, const float* B, float* C,
                   long long A_stride, long long B_stride, long long C_stride, long long tlo,
                   long long thi, cudaStream_t stream);
int runpair_tile_rows(const RunPairPlan* rp);
bool runpair_aligned(const RunPairPlan* rp, const void* A, const void* B, const void* C);


constexpr int kClusterSpan = 64;       /* max span of one A-offset cluster */
constexpr int kTileSmemCap = 100 * 1024;
constexpr int kTileThreads = 256;       /* CTAs that share an SM */
constexpr int kTileThreadsSolo = 1024;  /* a CTA alone on its SM (wide windows) */

struct Window {
    long long src;   /* element offset in B_vals of the window at tile row 0 */
    int soff;        /* shared-memory float offset */
    int len4;        /* 16-byte chunks */
};

struct TileArgs {
    const float* A;
    const float* B;
    float* C;
    const Window* win;
    const int2* terms;    /* (A slot offset, B window offset) in floats */
    const int* tptr;      /* [nC + 1] */
    int nA, nwin, nC, nterms;
    long long A_stride, C_stride, vrow0;
    int i_lo, ntiles, T, stage_floats;
};

__device__ __forceinline__ void cp_async16(uint32_t dst, const float* src)
{
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}

template <int R, int NT>
__global__ void __launch_bounds__(NT) tile_sum_kernel(TileArgs p)
{
    constexpr int kTileWarps = NT / 32;
    extern __shared__ __align__(16) float sm[];
    constexpr int T = 32 * R;
    int2* s_terms = (int2*)(sm + p.stage_floats);
    int* s_tptr = (int*)(s_terms + p.nterms);
    /* window table after the term lists, 8-byte aligned */
    Window* s_win = (Window*)(((uintptr_t)(s_tptr + p.nC + 1) + 7) & ~(uintptr_t)7);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    for (int t = tid; t < p.nterms; t += NT) s_terms[t] = p.terms[t];
    for (int c = tid; c <= p.nC; c += NT) s_tptr[c] = p.tptr[c];
    for (int w = tid; w < p.nwin; w += NT) s_win[w] = p.win[w];
    const uint32_t sbase = (uint32_t)__cvta_generic_to_shared(sm);

    for (int tile = blockIdx.x; tile < p.ntiles; tile += gridDim.x) {
        const long long t0 = (long long)p.i_lo + (long long)tile * T;
        __syncthreads();  /* previous tile's readers are done with sm */
        for (int a = warp; a < p.nA; a += kTileWarps) {
            const float* src = p.A + a * p.A_stride + (t0 - p.vrow0);
            for (int q = lane; q < T / 4; q += 32)
                cp_async16(sbase + (uint32_t)(a * T + 4 * q) * 4u, src + 4 * q);
        }
        for (int w = warp; w < p.nwin; w += kTileWarps) {
            const Window wd = s_win[w];
            const float* src = p.B + wd.src + t0;
            for (int q = lane; q < wd.len4; q += 32)
                cp_async16(sbase + (uint32_t)(wd.soff + 4 * q) * 4u, src + 4 * q);
        }
        asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
        __syncthreads();
        float* cbase = p.C + (t0 - p.vrow0) + lane;
        for (int c = warp; c < p.nC; c += kTileWarps) {
            float acc[R];
#pragma unroll
            for (int j = 0; j < R; ++j) acc[j] = 0.0f;
            const int q1 = s_tptr[c + 1];
            for (int q = s_tptr[c]; q < q1; ++q) {
                const int2 t = s_terms[q];
                const float* ua = sm + t.x + lane;
                const float* vb = sm + t.y + lane;
#pragma unroll
                for (int j = 0; j < R; ++j) acc[j] = mul_add_rn(acc[j], ua[32 * j], vb[32 * j]);
            }
            float* dst = cbase + (long long)c * p.C_stride;
#pragma unroll
            for (int j = 0; j < R; ++j) __stcs(dst + 32 * j, acc[j]);
        }
    }
}

}  // namespace dia

using namespace dia;

struct DiaSpmspmPlan {
    int n = 0, nA = 0, nB = 0, nC = 0;
    long long A_stride = 0, B_stride = 0, C_stride = 0, vrow0 = 0, b_vrow0 = 0;
    int b_lo = 0, b_hi = 0, rows_lo = 0, rows_hi = 0;
    std::vector<int> C_off, C_len;
    std::vector<long long> C_start;
    /* tiled path */
    int T = 0, i_lo = 0, i_hi = 0, nwin = 0, nterms = 0, stage_floats = 0, smem = 0;
    Window* d_win = nullptr;
    int2* d_terms = nullptr;
    int* d_tptr = nullptr;
    /* generic path (edge rows) */
    Term* d_gterms = nullptr;
    OutDesc* d_gouts = nullptr;
    int* d_offs = nullptr;   /* A | B | C offsets on the device */
    float avg_terms = -1.0f; /* pairs per output diagonal */
    RunPairPlan rp;          /* register-blocked path for run-structured offsets */
    /* edge rows run on this high-priority stream, concurrently with the
     * interior kernel on the caller's stream (they write disjoint rows);
     * executions of one plan that overlap on the host share it */
    cudaStream_t side = nullptr;
    cudaEvent_t fork = nullptr, join = nullptr;
};

namespace {

int plan_free(DiaSpmspmPlan* p)
{
    if (!p) return DIA_OK;
    runpair_plan_free(&p->rp);
    cudaFree(p->d_win);
    cudaFree(p->d_terms);
    cudaFree(p->d_tptr);
    cudaFree(p->d_gterms);
    cudaFree(p->d_gouts);
    cudaFree(p->d_offs);
    if (p->side) cudaStreamDestroy(p->side);
    if (p->fork) cudaEventDestroy(p->fork);
    if (p->join) cudaEventDestroy(p->join);
    delete p;
    return DIA_OK;
}

long long mod4(long long x) { return ((x % 4) + 4) % 4; }

}  // namespace


extern "C" int dia_spmspm_plan_create(int64_t n, const int* h_A_off, int nA, const int* h_B_off,
                                      int nB, int64_t A_stride, int64_t B_stride,
                                      int64_t C_stride, int64_t vrow0, int64_t nrows,
                                      int64_t b_vrow0, int64_t b_lo, int64_t b_hi,
                                      DiaSpmspmPlan** out)
{
    if (!out) return fail(DIA_ERR_INVALID, "dia_spmspm_plan_create: null plan pointer");
    *out = nullptr;
    if (n <= 0 || n + kTile >= (1LL << 31) || nA < 0 || nB < 0 || nrows < 0)
        return fail(DIA_ERR_INVALID, "dia_spmspm_plan_create: bad sizes");
    if (nrows > C_stride || nrows > A_stride || b_lo < b_vrow0 || b_hi > b_vrow0 + B_stride)
        return fail(DIA_ERR_INVALID, "dia_spmspm_plan_create: rows outside the buffers");
    int nc = 0;
    int64_t np = 0;
    int rc = dia_spmspm_symbolic((int)n, h_A_off, nA, h_B_off, nB, &nc, nullptr, nullptr,
                                 nullptr, &np, nullptr, nullptr, nullptr);
    if (rc) return rc;
    auto* P = new DiaSpmspmPlan();
    P->n = (int)n; P->nA = nA; P->nB = nB; P->nC = nc;
    P->A_stride = A_stride; P->B_stride = B_stride; P->C_stride = C_stride;
    P->vrow0 = vrow0; P->b_vrow0 = b_vrow0;
    P->b_lo = (int)std::max<int64_t>(b_lo, 0); P->b_hi = (int)std::min<int64_t>(b_hi, n);
    P->rows_lo = (int)vrow0; P->rows_hi = (int)std::min<int64_t>(vrow0 + nrows, n);
    P->C_off.resize(nc); P->C_len.resize(nc); P->C_start.resize(nc);
    P->avg_terms = nc > 0 ? (float)np / nc : -1.0f;
    std::vector<int> ptr(nc + 1), pa(std::max<int64_t>(np, 1)), pb(std::max<int64_t>(np, 1));
    rc = dia_spmspm_symbolic((int)n, h_A_off, nA, h_B_off, nB, &nc, P->C_off.data(),
                             P->C_len.data(), (int64_t*)P->C_start.data(), &np, ptr.data(),
                             pa.data(), pb.data());
    if (rc) { plan_free(P); return rc; }

    auto cuda = [&](cudaError_t e, const char* w) -> int {
        if (e == cudaSuccess) return (int)DIA_OK;
        plan_free(P);
        return cuda_fail(e, w);
    };
    /* device offsets + generic terms over the whole row block */
    const int ntot = nA + nB + nc;
    if ((rc = cuda(cudaMalloc(&P->d_offs, sizeof(int) * std::max(ntot, 1)), "cudaMalloc")))
        return rc;
    std::vector<int> offs;
    offs.insert(offs.end(), h_A_off, h_A_off + nA);
    offs.insert(offs.end(), h_B_off, h_B_off + nB);
    offs.insert(offs.end(), P->C_off.begin(), P->C_off.end());
    if ((rc = cuda(cudaMemcpy(P->d_offs, offs.data(), sizeof(int) * ntot, cudaMemcpyHostToDevice),
                   "cudaMemcpy")))
        return rc;
    if (nc > 0) {
        if ((rc = cuda(cudaMalloc(&P->d_gterms, sizeof(Term) * (size_t)nc * std::max(nA, 1)),
                       "cudaMalloc")) ||
            (rc = cuda(cudaMalloc(&P->d_gouts, sizeof(OutDesc) * nc), "cudaMalloc")))
            return rc;
        rc = build_generic_terms_rows(n, P->d_offs, nA, P->d_offs + nA, nB, P->d_offs + nA + nB,
                                      nc, A_stride, B_stride, b_vrow0, b_lo, b_hi, C_stride,
                                      vrow0, P->rows_lo, P->rows_hi, P->d_gterms, P->d_gouts, 0);
        if (rc) { plan_free(P); return rc; }
        if ((rc = cuda(cudaDeviceSynchronize(), "plan build"))) return rc;
    }

    /* run-pair path (stencils, bands): preferred when the offsets allow it */
    if (nc > 0 && np > 0 && nA > 0)
        runpair_plan_build(h_A_off, nA, h_B_off, nB, P->C_off.data(), nc, A_stride, B_stride,
                           C_stride, vrow0, b_vrow0, P->b_lo, P->b_hi, P->rows_lo, P->rows_hi,
                           &P->rp);
    /* tiled path: interior rows, where every term is in range */
    if (nc > 0 && np > 0 && nA > 0 && !P->rp.P) {
        const int dmin = *std::min_element(h_A_off, h_A_off + nA);
        const int dmax = *std::max_element(h_A_off, h_A_off + nA);
        long long lo = std::max<long long>(P->rows_lo, (long long)P->b_lo - dmin + 4);
        long long hi = std::min<long long>(P->rows_hi, (long long)P->b_hi - dmax - 4);
        lo = std::max<long long>(lo, 0);
        lo += mod4(vrow0 - lo);                    /* A slot loads 16-byte aligned */
        int dev = 0, smem_max = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&smem_max, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
        /* first try clusters of span <= kClusterSpan at two CTAs per SM; if
         * that does not fit, one cluster spanning all of A's offsets (one B
         * window per B diagonal, e.g. 32 scattered offsets in [-512, 512])
         * at one CTA per SM with up to all of the shared memory */
        for (int wide = 0; wide < 2 && !P->T; ++wide) {
            const int span = wide ? INT_MAX : kClusterSpan;
            const int cap = wide ? smem_max : std::min(smem_max, kTileSmemCap);
            /* clusters of A offsets */
            std::vector<int> ds(h_A_off, h_A_off + nA);
            std::sort(ds.begin(), ds.end());
            std::map<int, int> clus;                   /* offset -> cluster id */
            std::vector<int> cl_lo, cl_hi;
            for (int d : ds) {
                if (cl_lo.empty() || (long long)d - cl_lo.back() > span) {
                    cl_lo.push_back(d);
                    cl_hi.push_back(d);
                }
                cl_hi.back() = d;
                clus[d] = (int)cl_lo.size() - 1;
            }
            /* only tiles of >= 128 rows: with fewer rows per lane the per-term
             * overhead outweighs the shared-memory reuse (measured: a 27-point
             * stencil product ran slower at 64-row tiles than the generic
             * kernel) */
            for (int R : {8, 4}) {
                const int T = 32 * R;
                if (hi - lo < 2LL * T) continue;
                std::map<std::pair<int, int>, int> wid;
                std::vector<Window> win;
                std::vector<int2> terms;
                std::vector<int> tptr(nc + 1);
                int soff = nA * T;
                const long long align = mod4(b_vrow0 - lo);   /* start row offset alignment */
                std::vector<int> wstart;
                for (int c = 0; c < nc; ++c) {
                    tptr[c] = (int)terms.size();
                    for (int q = ptr[c]; q < ptr[c + 1]; ++q) {
                        const int a = pa[q], b = pb[q], da = h_A_off[a];
                        const int cl = clus[da];
                        auto key = std::make_pair(b, cl);
                        auto it = wid.find(key);
                        int w;
                        if (it == wid.end()) {
                            const long long s = cl_lo[cl] - mod4(cl_lo[cl] - align);
                            const long long len = (cl_hi[cl] + T - s + 3) / 4 * 4;
                            Window W;
                            W.src = (long long)b * B_stride - b_vrow0 + s;
                            W.soff = soff;
                            W.len4 = (int)(len / 4);
                            soff += (int)len;
                            w = (int)win.size();
                            win.push_back(W);
                            wstart.push_back((int)s);
                            wid[key] = w;
                        } else {
                            w = it->second;
                        }
                        terms.push_back(make_int2(a * T, win[w].soff + (da - wstart[w])));
                    }
                }
                tptr[nc] = (int)terms.size();
                const int smem = (soff * 4 + (int)terms.size() * 8 + (nc + 1) * 4 + 7) / 8 * 8 +
                                 (int)win.size() * (int)sizeof(Window);
                /* clustered: at least two CTAs per SM, so one tile's copies
                 * overlap another's products */
                if (smem > cap) continue;
                P->T = T;
                P->i_lo = (int)lo;
                P->i_hi = (int)(lo + (hi - lo) / T * T);
                P->nwin = (int)win.size();
                P->nterms = (int)terms.size();
                P->stage_floats = soff;
                P->smem = smem;
                if ((rc = cuda(cudaMalloc(&P->d_win, sizeof(Window) * win.size()), "cudaMalloc")) ||
                    (rc = cuda(cudaMalloc(&P->d_terms, sizeof(int2) * terms.size()), "cudaMalloc")) ||
                    (rc = cuda(cudaMalloc(&P->d_tptr, sizeof(int) * tptr.size()), "cudaMalloc")) ||
                    (rc = cuda(cudaMemcpy(P->d_win, win.data(), sizeof(Window) * win.size(),
                                          cudaMemcpyHostToDevice), "cudaMemcpy")) ||
                    (rc = cuda(cudaMemcpy(P->d_terms, terms.data(), sizeof(int2) * terms.size(),
                                          cudaMemcpyHostToDevice), "cudaMemcpy")) ||
                    (rc = cuda(cudaMemcpy(P->d_tptr, tptr.data(), sizeof(int) * tptr.size(),
                                          cudaMemcpyHostToDevice), "cudaMemcpy")))
                    return rc;
                break;
            }
        }
    }
    {
        int lo_prio = 0, hi_prio = 0;
        cudaDeviceGetStreamPriorityRange(&lo_prio, &hi_prio);
        if ((rc = cuda(cudaStreamCreateWithPriority(&P->side, cudaStreamNonBlocking, hi_prio),
                       "cudaStreamCreateWithPriority")) ||
            (rc = cuda(cudaEventCreateWithFlags(&P->fork, cudaEventDisableTiming),
                       "cudaEventCreate")) ||
            (rc = cuda(cudaEventCreateWithFlags(&P->join, cudaEventDisableTiming),
                       "cudaEventCreate"))) {
            plan_free(P);
            return rc;
        }
    }
    *out = P;
    return DIA_OK;
}

extern "C" int dia_spmspm_plan_info(const DiaSpmspmPlan* P, int* n_c, int* h_C_off,
                                    int* h_C_len, int64_t* h_C_start, int* tile_rows,
                                    int64_t* tiled_lo, int64_t* tiled_hi)
{
    if (!P) return fail(DIA_ERR_INVALID, "dia_spmspm_plan_info: null plan");
    if (n_c) *n_c = P->nC;
    for (int c = 0; c < P->nC; ++c) {
        if (h_C_off) h_C_off[c] = P->C_off[c];
        if (h_C_len) h_C_len[c] = P->C_len[c];
        if (h_C_start) h_C_start[c] = P->C_start[c];
    }
    if (P->rp.P) {
        if (tile_rows) *tile_rows = -runpair_tile_rows(&P->rp);   /* negative: run-pair kernel */
        if (tiled_lo) *tiled_lo = P->rp.i_lo;
        if (tiled_hi) *tiled_hi = P->rp.i_hi;
        return DIA_OK;
    }
    if (tile_rows) *tile_rows = P->T;
    if (tiled_lo) *tiled_lo = P->T ? P->i_lo : 0;
    if (tiled_hi) *tiled_hi = P->T ? P->i_hi : 0;
    return DIA_OK;
}

extern "C" int dia_spmspm_plan_execute(const DiaSpmspmPlan* P, const float* d_A_vals,
                                       const float* d_B_vals, float* d_C_vals, int64_t row_lo,
                                       int64_t row_hi, int use_tiles, cudaStream_t stream)
{
    if (!P) return fail(DIA_ERR_INVALID, "dia_spmspm_plan_execute: null plan");
    row_lo = std::max<int64_t>(row_lo, P->rows_lo);
    row_hi = std::min<int64_t>(row_hi, P->rows_hi);
    if (row_hi <= row_lo || P->nC == 0) return DIA_OK;
    if (!d_A_vals || !d_B_vals || !d_C_vals)
        return fail(DIA_ERR_INVALID, "dia_spmspm_plan_execute: null pointer");
    long long tlo = row_hi, thi = row_hi;
    int kind = 0;   /* interior kernel: 1 run-pair, 2 tiled */
    if (use_tiles && P->rp.P && runpair_aligned(&P->rp, d_A_vals, d_B_vals, d_C_vals)) {
        const long long T = runpair_tile_rows(&P->rp);
        const long long first = std::max<long long>(0, (row_lo - P->rp.i_lo + T - 1) / T);
        const long long last = (std::min<long long>(row_hi, P->rp.i_hi) - P->rp.i_lo) / T;
        if (last > first && row_lo < P->rp.i_hi) {
            tlo = P->rp.i_lo + first * T;
            thi = P->rp.i_lo + last * T;
            kind = 1;
        }
    } else if (use_tiles && P->T) {
        /* whole tiles inside both the interior and [row_lo, row_hi) */
        const long long first = std::max<long long>(0, (row_lo - P->i_lo + P->T - 1) / P->T);
        const long long last = (std::min<long long>(row_hi, P->i_hi) - P->i_lo) / P->T;
        if (last > first && row_lo < P->i_hi) {
            tlo = P->i_lo + first * P->T;
            thi = P->i_lo + last * P->T;
            kind = 2;
        }
    }
    const bool edges = tlo > row_lo || row_hi > thi;
    cudaStream_t es = stream;
    if (edges && kind && P->side) {
        DIA_TRY_CUDA(cudaEventRecord(P->fork, stream));
        DIA_TRY_CUDA(cudaStreamWaitEvent(P->side, P->fork, 0));
        es = P->side;
    }
    int rc = DIA_OK;
    const float* U = d_A_vals;
    if (tlo > row_lo)
        rc = launch_pair_sum(U, d_B_vals, d_C_vals, P->d_gouts, P->d_gterms, P->nC, (int)row_lo,
                             (int)tlo, false, es, P->avg_terms);
    if (rc == DIA_OK && row_hi > thi)
        rc = launch_pair_sum(U, d_B_vals, d_C_vals, P->d_gouts, P->d_gterms, P->nC, (int)thi,
                             (int)row_hi, false, es, P->avg_terms);
    if (es != stream) DIA_TRY_CUDA(cudaEventRecord(P->join, es));
    if (rc) return rc;
    if (kind == 1) {
        rc = runpair_launch(&P->rp, d_A_vals, d_B_vals, d_C_vals, P->A_stride, P->B_stride,
                            P->C_stride, tlo, thi, stream);
    } else if (kind == 2) {
        TileArgs a{};
        a.A = d_A_vals;
        a.B = d_B_vals;
        a.C = d_C_vals;
        a.win = P->d_win;
        a.terms = P->d_terms;
        a.tptr = P->d_tptr;
        a.nA = P->nA;
        a.nwin = P->nwin;
        a.nC = P->nC;
        a.nterms = P->nterms;
        a.A_stride = P->A_stride;
        a.C_stride = P->C_stride;
        a.vrow0 = P->vrow0;
        a.i_lo = (int)tlo;
        a.ntiles = (int)((thi - tlo) / P->T);
        a.T = P->T;
        a.stage_floats = P->stage_floats;
        auto pick = [&](bool solo) -> const void* {
            if (solo)
                return P->T == 256 ? (const void*)tile_sum_kernel<8, kTileThreadsSolo>
                     : P->T == 128 ? (const void*)tile_sum_kernel<4, kTileThreadsSolo>
                     : P->T == 64 ? (const void*)tile_sum_kernel<2, kTileThreadsSolo>
                                  : (const void*)tile_sum_kernel<1, kTileThreadsSolo>;
            return P->T == 256 ? (const void*)tile_sum_kernel<8, kTileThreads>
                 : P->T == 128 ? (const void*)tile_sum_kernel<4, kTileThreads>
                 : P->T == 64 ? (const void*)tile_sum_kernel<2, kTileThreads>
                              : (const void*)tile_sum_kernel<1, kTileThreads>;
        };
        const void* k = pick(false);
        DIA_TRY_CUDA(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          P->smem));
        int per_sm = 0;
        DIA_TRY_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k, kTileThreads,
                                                                   P->smem));
        /* a CTA that has its SM to itself runs 32 warps: with 8 the
         * shared-memory latency of the products is exposed (measured on
         * config 3: 12.5 % warps active, 37 % issue) */
        int nt = kTileThreads;
        if (per_sm <= 1) {
            k = pick(true);
            nt = kTileThreadsSolo;
            DIA_TRY_CUDA(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                              P->smem));
            per_sm = 1;
        }
        /* clustered form: one CTA per tile (config 2: 0.081 ms against
         * 0.083 with a persistent grid); the 1024-thread form keeps one
         * persistent CTA per SM (config 3: 0.585 against 0.597 ms) */
        const int grid = nt == kTileThreads ? a.ntiles
                                            : (int)std::min<long long>(a.ntiles,
                                                  (long long)std::max(per_sm, 1) * num_sms());
        void* args[] = {&a};
        DIA_TRY_CUDA(cudaLaunchKernel(k, grid, nt, args, P->smem, stream));
    }
    if (es != stream) DIA_TRY_CUDA(cudaStreamWaitEvent(stream, P->join, 0));
    return rc;
}

extern "C" int dia_spmspm_plan_destroy(DiaSpmspmPlan* P) { return plan_free(P); }
