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
 * then owns 4 consecutive rows of one block: W x 4 accumulators in
 * registers, the P x 4 A values of a run pair loaded once (float4), and for
 * each B diagonal of the run one aligned 12-value window (three float4
 * loads) that serves all P shifted uses.  Every register index is a
 * compile-time constant (the window's alignment shift is a uniform switch).
 * That is about 2.5 instructions per product instead of the ~10 of the
 * generic pair-sum kernel.
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
constexpr int kRpRows = kRpThreads * 4;   /* rows per tile */

struct RunPairDesc {
    long long a_elem;   /* A element offset of (first A diagonal of the run, row 0) */
    long long b_elem;   /* B element offset of (first B diagonal, row 0) + alpha - shift */
    int shift;          /* (row + alpha - b_vrow0) mod 4 at tile-aligned rows */
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

template <int P, int Q, int NL, int S>
__device__ __forceinline__ void rp_body(float (&acc)[P + Q - 1][4], const float (&a)[P][4],
                                        const float (&raw)[Q][4 * NL])
{
#pragma unroll
    for (int u = 0; u < P; ++u)
#pragma unroll
        for (int v = 0; v < Q; ++v)
#pragma unroll
            for (int j = 0; j < 4; ++j)
                acc[u + v][j] = mul_add_rn(acc[u + v][j], a[u][j], raw[v][S + u + j]);
}

template <int P, int Q>
__global__ void __launch_bounds__(kRpThreads) runpair_kernel(RpArgs p)
{
    constexpr int W = P + Q - 1;
    constexpr int NL = (3 + (P - 1) + 4 + 3) / 4;   /* float4 loads per B window */
    const long long items = (long long)p.nblk * p.ntiles;
    for (long long it = blockIdx.x; it < items; it += gridDim.x) {
        const int k = (int)(it % p.nblk);
        const long long i = (long long)p.i_lo + (it / p.nblk) * kRpRows + 4 * threadIdx.x;
        const RunBlock bk = p.blks[k];
        float acc[W][4];
#pragma unroll
        for (int s = 0; s < W; ++s)
#pragma unroll
            for (int j = 0; j < 4; ++j) acc[s][j] = 0.0f;
        for (int r = bk.rp0; r < bk.rp1; ++r) {
            const RunPairDesc d = p.rps[r];
            float a[P][4];
#pragma unroll
            for (int u = 0; u < P; ++u) {
                const float4 x = __ldg((const float4*)(p.A + d.a_elem + u * p.A_stride + i));
                a[u][0] = x.x; a[u][1] = x.y; a[u][2] = x.z; a[u][3] = x.w;
            }
            /* L1 wavefronts of these overlapping window loads bound this
             * kernel (ncu: L1 throughput 93 % of peak on config 5); loading
             * the last float4 only when the shift needs it measured slower */
            float raw[Q][4 * NL];
#pragma unroll
            for (int v = 0; v < Q; ++v)
#pragma unroll
                for (int m = 0; m < NL; ++m) {
                    const float4 x =
                        __ldg((const float4*)(p.B + d.b_elem + v * p.B_stride + i + 4 * m));
                    raw[v][4 * m] = x.x; raw[v][4 * m + 1] = x.y;
                    raw[v][4 * m + 2] = x.z; raw[v][4 * m + 3] = x.w;
                }
            switch (d.shift) {
                case 0: rp_body<P, Q, NL, 0>(acc, a, raw); break;
                case 1: rp_body<P, Q, NL, 1>(acc, a, raw); break;
                case 2: rp_body<P, Q, NL, 2>(acc, a, raw); break;
                default: rp_body<P, Q, NL, 3>(acc, a, raw); break;
            }
        }
#pragma unroll
        for (int s = 0; s < W; ++s)
            __stcs((float4*)(p.C + bk.c_elem + s * p.C_stride + i),
                   make_float4(acc[s][0], acc[s][1], acc[s][2], acc[s][3]));
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
    long long lo = std::max<long long>(rows_lo, (long long)b_lo - dmin + 16);
    long long hi = std::min<long long>(rows_hi, (long long)b_hi - dmax - 16);
    lo = std::max<long long>(lo, 0);
    lo += ((vrow0 - lo) % 4 + 4) % 4;
    if (hi - lo < 2LL * kRpRows) return false;
    rp->P = P;
    rp->Q = Q;
    rp->i_lo = (int)lo;
    rp->i_hi = (int)(lo + (hi - lo) / kRpRows * kRpRows);
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
            d.shift = (int)(((lo + alpha - b_vrow0) % 4 + 4) % 4);
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
    a.ntiles = (int)((thi - tlo) / kRpRows);
    if (a.ntiles <= 0) return DIA_OK;
    const void* k = rp->P == 2 ? (const void*)runpair_kernel<2, 2>
                  : rp->P == 3 ? (const void*)runpair_kernel<3, 3>
                  : rp->P == 4 ? (const void*)runpair_kernel<4, 4>
                               : (const void*)runpair_kernel<5, 5>;
    const long long items = (long long)a.nblk * a.ntiles;
    const int grid = (int)std::min<long long>(items, persistent_blocks(k, 0));
    void* args[] = {&a};
    DIA_TRY_CUDA(cudaLaunchKernel(k, grid, kRpThreads, args, 0, stream));
    return DIA_OK;
}

int runpair_tile_rows() { return kRpRows; }

}  // namespace dia
