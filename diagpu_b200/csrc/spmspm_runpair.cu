/*
 * spmspm_runpair.cu -- register-blocked SpMSpM for run-structured offsets.
 *
 * Stencil and band matrices have offsets that come in runs of consecutive
 * values (the 27-point stencil: nine runs of three).  If every run of A has
 * length P and every run of B length Q, each pair of runs
 *     A run [alpha, alpha+P) x B run [beta, beta+Q)
 * is a small dense band product landing on the W = P+Q-1 consecutive output
 * diagonals starting at alpha+beta:
 *     C[alpha+beta+s][i] += sum_{u+v=s} A[alpha+u][i] * B[beta+v][i+alpha+u].
 * When run pairs with different alpha+beta never overlap, the outputs split
 * into blocks of W diagonals, each fed by a list of run pairs.  A thread
 * owns R consecutive rows of one block (R = 8 for runs of 2 or 3, 4 for
 * longer runs): W x R accumulators in registers and the P x R A values of a
 * run pair, loaded as one aligned R-float vector per diagonal.
 *
 * The B values a thread needs for one B diagonal are the R + P - 1
 * consecutive rows i+alpha .. i+alpha+R+P-2: a window that starts D rows
 * into an aligned R-row chunk and spills into the next chunk (or two).  The
 * lanes of a warp own consecutive chunks, so each lane loads only one
 * aligned chunk (one fully coalesced vector load for the warp) and takes
 * the few values that lie in its neighbours' chunks with warp shuffles; the
 * lanes at the warp's two ends load the chunk past the warp themselves.
 * Loading overlapping windows instead moved 2-3 times the bytes through
 * the L1 data pipe, which bounded the kernel there (ncu: L1 at 93-97 % of
 * peak with DRAM at 28-37 %).  D is uniform per run pair, so every register
 * index is a compile-time constant (a uniform switch over D).
 *
 * Summation order: the run pairs of a block are sorted by alpha, and inside
 * a pair u ascends, so every output accumulates its terms in ascending A
 * offset -- the order of the reference CPU oracle
 * (spmspm/bench_spmspm.cu:392-403) when A's offsets are stored ascending,
 * which the planner requires.  Multiply and add are rounded separately:
 * results are bit-identical to the generic path.
 */
#include <algorithm>
#include <map>
#include <vector>

#include "../../include/diagpu_b200.h"
#include "dia_core.cuh"

namespace dia {

constexpr int kRpThreads = 256;

/* rows per thread: 8 for runs of 2 or 3, 4 for longer runs (registers) */
template <int P>
struct RpRows {
    static constexpr int value = P <= 3 ? 8 : 4;
};
template <int P>
__host__ __device__ constexpr int rp_tile_rows() { return kRpThreads * RpRows<P>::value; }

struct RunPairDesc {
    long long a_elem;   /* A element offset of (first A diagonal of the run, row 0) */
    long long b_elem;   /* B element offset of (first B diagonal, row 0) + alpha - shift */
    int shift;          /* (row + alpha - b_vrow0) mod R at tile-aligned rows */
    int pad;
};

struct RunBlock {
    long long c_elem;   /* C element offset of (first output diagonal, row 0) */
    int rp0, rp1;
};

struct RpArgs {
    const float* A;
    const float* B;
    float* C;
    const RunBlock* blks;
    const RunPairDesc* rps;
    long long A_stride, B_stride, C_stride;
    int nblk, i_lo, ntiles;
};

/* aligned R-float vector load (read-only path) and streaming store */
template <int R>
__device__ __forceinline__ void vload(float (&r)[R], const float* p);
template <>
__device__ __forceinline__ void vload<4>(float (&r)[4], const float* p)
{
    const float4 x = __ldg((const float4*)p);
    r[0] = x.x; r[1] = x.y; r[2] = x.z; r[3] = x.w;
}
template <>
__device__ __forceinline__ void vload<8>(float (&r)[8], const float* p)
{
    asm volatile("ld.global.nc.v8.f32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=f"(r[0]), "=f"(r[1]), "=f"(r[2]), "=f"(r[3]), "=f"(r[4]), "=f"(r[5]),
                   "=f"(r[6]), "=f"(r[7])
                 : "l"(p));
}
template <int R>
__device__ __forceinline__ void vstore_cs(float* p, const float (&r)[R]);
template <>
__device__ __forceinline__ void vstore_cs<4>(float* p, const float (&r)[4])
{
    __stcs((float4*)p, make_float4(r[0], r[1], r[2], r[3]));
}
template <>
__device__ __forceinline__ void vstore_cs<8>(float* p, const float (&r)[8])
{
    asm volatile("st.global.cs.v8.f32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};"
                 ::"l"(p), "f"(r[0]), "f"(r[1]), "f"(r[2]), "f"(r[3]), "f"(r[4]), "f"(r[5]),
                   "f"(r[6]), "f"(r[7])
                 : "memory");
}

/* Window positions [D, D+L) relative to the aligned chunk start; chunk
 * q = p / R.  The lane loads chunk `own` and shuffles the rest in: pick the
 * chunk that leaves the fewest positions outside it. */
__host__ __device__ constexpr int rp_outside(int D, int L, int R, int c)
{
    int n = 0;
    for (int p = D; p < D + L; ++p) n += (p / R != c);
    return n;
}
__host__ __device__ constexpr int rp_own(int D, int L, int R)
{
    int best = 0;
    for (int c = 1; c <= (D + L - 1) / R; ++c)
        if (rp_outside(D, L, R, c) < rp_outside(D, L, R, best)) best = c;
    return best;
}

/* One run pair on R consecutive rows.  bp points at B row (i + alpha - D)
 * of the run's first B diagonal, an aligned chunk start. */
template <int P, int Q, int R, int D>
__device__ __forceinline__ void rp_body(float (&acc)[P + Q - 1][R], const float (&a)[P][R],
                                        const float* __restrict__ bp, long long B_stride,
                                        int lane)
{
    constexpr int L = P + R - 1;                 /* window length */
    constexpr int NQ = (D + L - 1) / R + 1;      /* chunks the window touches */
    constexpr int OWN = rp_own(D, L, R);
    /* v descends outermost and u ascends inside it, so every output
     * (u + v fixed) still takes its terms in ascending u; only one B
     * window is live at a time */
#pragma unroll
    for (int v = Q - 1; v >= 0; --v) {
        const float* cp = bp + v * B_stride;
        float w[L];
        float own[R];
        vload<R>(own, cp + OWN * R);
#pragma unroll
        for (int q = 0; q < NQ; ++q) {
            if (q == OWN) {
#pragma unroll
                for (int p = D; p < D + L; ++p)
                    if (p / R == q) w[p - D] = own[p % R];
                continue;
            }
            /* lanes whose neighbour lane + (q - OWN) lies outside the warp
             * load that chunk themselves */
            const int src = lane + (q - OWN);
            const bool outside = src < 0 || src > 31;
            float fx[R];
#pragma unroll
            for (int k = 0; k < R; ++k) fx[k] = 0.0f;
            if (outside) vload<R>(fx, cp + q * R);
#pragma unroll
            for (int p = D; p < D + L; ++p)
                if (p / R == q) {
                    const float sh = __shfl_sync(0xffffffffu, own[p % R], src & 31);
                    w[p - D] = outside ? fx[p % R] : sh;
                }
        }
#pragma unroll
        for (int u = 0; u < P; ++u)
#pragma unroll
            for (int j = 0; j < R; ++j)
                acc[u + v][j] = mul_add_rn(acc[u + v][j], a[u][j], w[u + j]);
    }
}

/* D is uniform per run pair: one switch picks the body compiled for it
 * (both branches are compiled for every R, hence the D % R in the R = 8
 * cases, which keeps the R = 4 instantiations' template arguments valid) */
template <int P, int Q, int R>
__device__ __forceinline__ void rp_dispatch(float (&acc)[P + Q - 1][R], const float (&a)[P][R],
                                            const float* bp, long long B_stride, int lane,
                                            int D)
{
    if (R == 8) {
        switch (D) {
            case 0: rp_body<P, Q, R, 0>(acc, a, bp, B_stride, lane); break;
            case 1: rp_body<P, Q, R, 1>(acc, a, bp, B_stride, lane); break;
            case 2: rp_body<P, Q, R, 2>(acc, a, bp, B_stride, lane); break;
            case 3: rp_body<P, Q, R, 3>(acc, a, bp, B_stride, lane); break;
            case 4: rp_body<P, Q, R, 4 % R>(acc, a, bp, B_stride, lane); break;
            case 5: rp_body<P, Q, R, 5 % R>(acc, a, bp, B_stride, lane); break;
            case 6: rp_body<P, Q, R, 6 % R>(acc, a, bp, B_stride, lane); break;
            default: rp_body<P, Q, R, 7 % R>(acc, a, bp, B_stride, lane); break;
        }
    } else {
        switch (D) {
            case 0: rp_body<P, Q, R, 0>(acc, a, bp, B_stride, lane); break;
            case 1: rp_body<P, Q, R, 1>(acc, a, bp, B_stride, lane); break;
            case 2: rp_body<P, Q, R, 2>(acc, a, bp, B_stride, lane); break;
            default: rp_body<P, Q, R, 3>(acc, a, bp, B_stride, lane); break;
        }
    }
}

template <int P, int Q>
__global__ void __launch_bounds__(kRpThreads) runpair_kernel(RpArgs p)
{
    constexpr int W = P + Q - 1;
    constexpr int R = RpRows<P>::value;
    const int lane = threadIdx.x & 31;
    const long long items = (long long)p.nblk * p.ntiles;
    for (long long it = blockIdx.x; it < items; it += gridDim.x) {
        const int k = (int)(it % p.nblk);
        const long long i =
            (long long)p.i_lo + (it / p.nblk) * rp_tile_rows<P>() + R * threadIdx.x;
        const RunBlock bk = p.blks[k];
        float acc[W][R];
#pragma unroll
        for (int s = 0; s < W; ++s)
#pragma unroll
            for (int j = 0; j < R; ++j) acc[s][j] = 0.0f;
        for (int r = bk.rp0; r < bk.rp1; ++r) {
            const RunPairDesc d = p.rps[r];
            float a[P][R];
#pragma unroll
            for (int u = 0; u < P; ++u) vload<R>(a[u], p.A + d.a_elem + u * p.A_stride + i);
            rp_dispatch<P, Q, R>(acc, a, p.B + d.b_elem + i, p.B_stride, lane, d.shift);
        }
#pragma unroll
        for (int s = 0; s < W; ++s) vstore_cs<R>(p.C + bk.c_elem + s * p.C_stride + i, acc[s]);
    }
}

/* ------------------------------------------------------------------ host */

struct RunPairPlan {
    int P = 0, Q = 0, nblk = 0, i_lo = 0, i_hi = 0;
    RunBlock* d_blks = nullptr;
    RunPairDesc* d_rps = nullptr;
};

static bool runs_of(const int* off, int n, int& len, std::vector<int>& starts)
{
    starts.clear();
    if (n == 0) return false;
    for (int i = 1; i < n; ++i)
        if (off[i] <= off[i - 1]) return false;   /* storage must be ascending */
    int cur = 1;
    len = -1;
    starts.push_back(0);
    for (int i = 1; i <= n; ++i) {
        if (i < n && off[i] == off[i - 1] + 1) {
            ++cur;
            continue;
        }
        if (len < 0) len = cur;
        if (cur != len) return false;
        if (i < n) starts.push_back(i);
        cur = 1;
    }
    return true;
}

static bool instantiated(int P, int Q) { return P == Q && P >= 2 && P <= 5; }

static long long rp_rows_of(int P)
{
    return P == 2 ? rp_tile_rows<2>() : P == 3 ? rp_tile_rows<3>()
         : P == 4 ? rp_tile_rows<4>() : rp_tile_rows<5>();
}

/* Builds the run-pair plan; returns false (and leaves *rp empty) when the
 * offsets do not have the structure or the interior is too small. */
bool runpair_plan_build(const int* hA, int nA, const int* hB, int nB, const int* hC, int nC,
                        long long A_stride, long long B_stride, long long C_stride,
                        long long vrow0, long long b_vrow0, int b_lo, int b_hi, int rows_lo,
                        int rows_hi, RunPairPlan* rp)
{
    int P, Q;
    std::vector<int> ra, rb;
    if (!runs_of(hA, nA, P, ra) || !runs_of(hB, nB, Q, rb) || !instantiated(P, Q)) return false;
    const int W = P + Q - 1;
    std::map<int, int> cidx;
    for (int c = 0; c < nC; ++c) cidx[hC[c]] = c;
    std::map<long long, std::vector<std::pair<int, int>>> blocks;   /* alpha+beta -> run pairs */
    for (int x : ra)
        for (int y : rb) blocks[(long long)hA[x] + hB[y]].push_back({x, y});
    long long prev = 0;
    bool first = true;
    for (auto& kv : blocks) {
        if (!first && kv.first - prev < W) return false;   /* blocks must not overlap */
        first = false;
        prev = kv.first;
        for (int s = 0; s < W; ++s)
            if (!cidx.count((int)(kv.first + s))) return false;
        if (cidx[(int)kv.first] + W - 1 != cidx[(int)(kv.first + W - 1)]) return false;
    }
    const int dmin = *std::min_element(hA, hA + nA), dmax = *std::max_element(hA, hA + nA);
    const long long T = rp_rows_of(P), R = T / kRpThreads;
    /* the chunks a thread loads reach at most R - 1 rows before its first
     * B row and 3R past its last */
    if (A_stride % R || B_stride % R || C_stride % R) return false;
    long long lo = std::max<long long>(rows_lo, (long long)b_lo - dmin + 4 * R);
    long long hi = std::min<long long>(rows_hi, (long long)b_hi - dmax - 4 * R);
    lo = std::max<long long>(lo, 0);
    lo += ((vrow0 - lo) % R + R) % R;
    if (hi - lo < 2LL * T) return false;
    rp->P = P;
    rp->Q = Q;
    rp->i_lo = (int)lo;
    rp->i_hi = (int)(lo + (hi - lo) / T * T);
    std::vector<RunBlock> bl;
    std::vector<RunPairDesc> ds;
    for (auto& kv : blocks) {
        auto pairs = kv.second;
        std::sort(pairs.begin(), pairs.end(),
                  [&](const std::pair<int, int>& x, const std::pair<int, int>& y) {
                      return hA[x.first] < hA[y.first];
                  });
        RunBlock b;
        b.c_elem = (long long)cidx[(int)kv.first] * C_stride - vrow0;
        b.rp0 = (int)ds.size();
        for (auto& pr : pairs) {
            const long long alpha = hA[pr.first];
            RunPairDesc d;
            d.shift = (int)(((lo + alpha - b_vrow0) % R + R) % R);
            d.a_elem = (long long)pr.first * A_stride - vrow0;
            d.b_elem = (long long)pr.second * B_stride - b_vrow0 + alpha - d.shift;
            d.pad = 0;
            ds.push_back(d);
        }
        b.rp1 = (int)ds.size();
        bl.push_back(b);
    }
    rp->nblk = (int)bl.size();
    if (cudaMalloc(&rp->d_blks, sizeof(RunBlock) * bl.size()) != cudaSuccess) return false;
    if (cudaMalloc(&rp->d_rps, sizeof(RunPairDesc) * ds.size()) != cudaSuccess) {
        cudaFree(rp->d_blks);
        rp->d_blks = nullptr;
        return false;
    }
    cudaMemcpy(rp->d_blks, bl.data(), sizeof(RunBlock) * bl.size(), cudaMemcpyHostToDevice);
    cudaMemcpy(rp->d_rps, ds.data(), sizeof(RunPairDesc) * ds.size(), cudaMemcpyHostToDevice);
    return true;
}

void runpair_plan_free(RunPairPlan* rp)
{
    cudaFree(rp->d_blks);
    cudaFree(rp->d_rps);
    rp->d_blks = nullptr;
    rp->d_rps = nullptr;
    rp->P = 0;
}

/* Rows [tlo, thi) (multiples of the tile inside [i_lo, i_hi)). */
int runpair_launch(const RunPairPlan* rp, const float* A, const float* B, float* C,
                   long long A_stride, long long B_stride, long long C_stride, long long tlo,
                   long long thi, cudaStream_t stream)
{
    RpArgs a{};
    a.A = A;
    a.B = B;
    a.C = C;
    a.blks = rp->d_blks;
    a.rps = rp->d_rps;
    a.A_stride = A_stride;
    a.B_stride = B_stride;
    a.C_stride = C_stride;
    a.nblk = rp->nblk;
    a.i_lo = (int)tlo;
    a.ntiles = (int)((thi - tlo) / rp_rows_of(rp->P));
    if (a.ntiles <= 0) return DIA_OK;
    const void* k = rp->P == 2 ? (const void*)runpair_kernel<2, 2>
                  : rp->P == 3 ? (const void*)runpair_kernel<3, 3>
                  : rp->P == 4 ? (const void*)runpair_kernel<4, 4>
                               : (const void*)runpair_kernel<5, 5>;
    const long long items = (long long)a.nblk * a.ntiles;
    /* one CTA per work item, not a persistent grid: the block scheduler
     * then balances the items, including when another stream's kernel (a
     * halo exchange) holds SMs while this one starts; a persistent grid
     * with a fixed share of items per CTA measured 14.2-15.1 ms on config 5
     * against 12.9 ms this way */
    const int grid = (int)std::min<long long>(items, 0x7fffffffLL);
    void* args[] = {&a};
    DIA_TRY_CUDA(cudaLaunchKernel(k, grid, kRpThreads, args, 0, stream));
    return DIA_OK;
}

int runpair_tile_rows(const RunPairPlan* rp) { return (int)rp_rows_of(rp->P); }

/* The kernel's vector loads and stores need buffers aligned to R floats. */
bool runpair_aligned(const RunPairPlan* rp, const void* A, const void* B, const void* C)
{
    const uintptr_t m = (uintptr_t)(4 * (rp_rows_of(rp->P) / kRpThreads)) - 1;
    return (((uintptr_t)A | (uintptr_t)B | (uintptr_t)C) & m) == 0;
}

}  // namespace dia
