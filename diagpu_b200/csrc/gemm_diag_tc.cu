/*
 * gemm_diag_tc.cu -- tcgen05 TF32 dense-band kernels for gemm_diag.
 *
 * Two kernels compute the same tiles: gemm_diag_ws_kernel (further down:
 * TMA-fed and warp-specialised, the default) and gemm_diag_tc_kernel
 * (below: operands built by 4-byte cp.async walks), used when TMA cannot
 * address the operands (n % 4 != 0, unaligned bases, > 256 diagonals).
 *
 * When A and B are contiguous bands (offsets a_lo..a_lo+P-1, b_lo..b_lo+Q-1),
 * a tile of 128 consecutive rows of C = A*B is a dense product
 *     C[r0:r0+128, cols] = A[r0:r0+128, K] * B[K, cols]
 * over the K = 127+P columns the tile's A rows touch.  gemm_diag_tc_kernel:
 *   - splits K into 32-column chunks; for chunk j it builds, in shared
 *     memory, the dense 128x32 slice of A and the (31+Q, padded to 16)x32
 *     slice of B in the K-major 128-byte-swizzled layout the tensor core
 *     reads (one 128-byte row per operand row, 8-row atoms).  Each warp walks one
 *     stored diagonal per instruction, so every global load is a coalesced
 *     run of consecutive rows; the tensor core reads the fp32 bits as TF32
 *     (low 13 mantissa bits ignored);
 *   - one thread issues four tcgen05.mma.kind::tf32 (K = 8 each) per chunk,
 *     accumulating into a 128 x 384 fp32 tile in tensor memory (zeroed
 *     first), chunk j landing at TMEM column 32*j; five operand stages,
 *     three chunks' copies in flight while the previous chunk's MMAs run,
 *     and tcgen05.commit -> mbarrier tells the builders when a stage is
 *     free again;
 *   - the epilogue copies the accumulator to a shared-memory tile
 *     (tcgen05.ld 32x32b.x32; the tile overlays the operand stages) and then
 *     writes each output diagonal's 128 rows as coalesced runs, overwriting
 *     (beta = 0) or adding to (beta = 1) the caller's HM-packed C.
 * Persistent CTAs, one per SM (the shared-memory request keeps two CTAs
 * from sharing an SM and so from competing for its tensor memory).  No TMA
 * and no multicast.  Every mbarrier wait is bounded: on timeout the kernel
 * records DIA_TC_TIMEOUT in a device status word (dia_device_status), stops
 * issuing, drains, frees its tensor memory and returns.
 *
 * Reference: gemm_diag_kernel (gemm_diag/gemm_diag.cu:119-329) computes the
 * same product with FP32 SIMT and global atomicAdd; this path computes in
 * TF32 (relative L2 within 5e-3 of an fp64 accumulation).
 */
#include <algorithm>
#include <cstdint>

#include <cuda.h>

#include "../../include/diagpu_b200.h"
#include "dia_core.cuh"

namespace dia {

constexpr int kTcRows = 128;        /* M of the MMA: rows per tile */
constexpr int kTcK = 32;            /* columns per K-chunk */
constexpr int kTcThreads = 512;
constexpr int kWarps = kTcThreads / 32;
constexpr int kStages = 5;          /* operand stages */
constexpr int kAhead = kStages - 2; /* chunks whose copies are in flight */
constexpr int kTcMaxDiags = 257;    /* P + Q - 1 */
constexpr int kECols = 384;         /* accumulator columns copied out */
constexpr int kEPitch = kECols + 1; /* odd pitch: conflict-free rows and diagonals */
constexpr int kEpiBytes = kTcRows * kEPitch * 4;
constexpr uint32_t kTmemCols = 512;
/* A walks: m0 = warp - 31 + lane spans [-31, kWarps - 1 + 0]; iterations
 * until every m in [0, 128) is covered */
constexpr int kAIters = (kTcRows + 31 + kWarps - 1) / kWarps;
constexpr int kMaxSmem = 227 * 1024;   /* opt-in dynamic shared memory per CTA */
constexpr long long kWaitLimit = 1LL << 26;

static __device__ unsigned int g_device_status;

struct TcArgs {
    const float* DA;
    const float* DB;
    float* C;
    const int* C_offsets;
    const int* C_lens;
    const int* k_to_idx;
    int n, P, Q, a_lo, b_lo;
    int nchunks, nmma;   /* K-chunks per tile, MMA N (B rows per chunk) */
    int ntiles, beta;
};

__device__ __forceinline__ uint32_t smem_u32(const void* p)
{
    return (uint32_t)__cvta_generic_to_shared(p);
}


/* byte offset of element (r, k) in a K-major operand slice of 32 K-columns
 * (one 128-byte row per r) with the 128-byte swizzle: 8-row atoms of 1024
 * bytes; within an atom the 16-byte chunk index is XORed with r % 8.  A
 * warp's copy writes one stored diagonal, cells (m0 + l, k0 + l); without
 * the swizzle those land in 8 banks (4-way conflicts), with it they spread
 * over the banks. */
__device__ __forceinline__ uint32_t kmajor_off(int r, int k)
{
    return (uint32_t)((r >> 3) * 1024 + (r & 7) * 128 + ((((k >> 2) ^ r) & 7) << 4) +
                      (k & 3) * 4);
}

/* UMMA shared-memory descriptor, K-major with 128-byte swizzle: SBO = 1024
 * bytes between 8-row atoms, LBO unused (1), sm_100 descriptor version 1. */
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr)
{
    uint64_t d = 0;
    d |= (uint64_t)((addr >> 4) & 0x3FFF);
    d |= (uint64_t)1 << 16;                          /* LBO (unused when swizzled) */
    d |= (uint64_t)((1024u >> 4) & 0x3FFF) << 32;   /* SBO */
    d |= (uint64_t)1 << 46;                          /* descriptor version */
    d |= (uint64_t)2 << 61;                          /* SWIZZLE_128B */
    return d;
}

/* one 4-byte cp.async into shared memory when `store`; `val` false copies
 * nothing from global memory and zero-fills the cell */
__device__ __forceinline__ void cp_async4(uint32_t dst, const float* src, bool store, bool val)
{
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %2, 0;\n\t"
        "@p cp.async.ca.shared.global [%0], [%1], 4, %3;\n\t}"
        ::"r"(dst), "l"(src), "r"((int)store), "r"(val ? 4 : 0) : "memory");
}

__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity)
{
    for (long long it = 0; it < kWaitLimit; ++it) {
        uint32_t ok;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(ok)
            : "r"(bar), "r"(parity)
            : "memory");
        if (ok) return true;
    }
    return false;
}

__global__ void __launch_bounds__(kTcThreads, 1) gemm_diag_tc_kernel(TcArgs a)
{
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    /* swizzle atoms must sit on 1024-byte boundaries of the shared window */
    unsigned char* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int a_bytes = kTcRows * kTcK * 4;          /* 16 KB */
    const int b_bytes = a.nmma * kTcK * 4;           /* <= 32 KB */
    /* the operand stages and the epilogue tile share the same bytes: the
     * stages are idle once a tile's MMAs have completed */
    const int st_bytes = a_bytes + b_bytes;
    auto a_stage = [&](int s) { return smem + s * st_bytes; };
    auto b_stage = [&](int s) { return smem + s * st_bytes + a_bytes; };
    float* etile = (float*)smem;                                         /* 128 x kEPitch */
    long long* kbase = (long long*)(smem + max(kEpiBytes, kStages * st_bytes));
    int* klo = (int*)(kbase + kTcMaxDiags);
    int* khi = klo + kTcMaxDiags;
    __shared__ __align__(8) unsigned long long mbar[kStages];
    __shared__ uint32_t s_tmem;

    const int nk = a.P + a.Q - 1;
    for (int kk = tid; kk < nk; kk += kTcThreads) {
        const int k = a.a_lo + a.b_lo + kk;
        const int ki = (k > -a.n && k < a.n) ? a.k_to_idx[k + a.n - 1] : -1;
        if (ki >= 0) {
            const int m = min(k, 0);
            kbase[kk] = (long long)a.C_offsets[ki] + m;
            klo[kk] = -m;
            khi[kk] = a.C_lens[ki] - m;
        } else {
            kbase[kk] = 0;
            klo[kk] = 1;
            khi[kk] = 0;
        }
    }
    if (tid == 0) {
        for (int s = 0; s < kStages; ++s)
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(&mbar[s])));
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     ::"r"(smem_u32(&s_tmem)), "r"(kTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = s_tmem;

    const uint32_t idesc = (1u << 4) | (2u << 7) | (2u << 10) |
                           ((uint32_t)(a.nmma >> 3) << 17) | ((uint32_t)(kTcRows >> 4) << 24);
    const int tm_cols = kTcK * (a.nchunks - 1) + a.nmma;
    /* per stage: bit s of `phase` = parity to wait for, of `pending` = MMAs
     * committed and not yet waited for (bit masks keep them in registers) */
    uint32_t phase = 0, pending = 0;
    bool ok = true;

    /* copy walks: lane l of warp w starts at operand row w - 31 + l; bit it
     * of a_tile / b_tile says whether iteration it lands inside the A / B
     * slice (the same for every chunk of every tile) */
    const int m0 = warp - 31 + lane;
    uint32_t a_tile = 0, b_tile = 0;
    const int b_iters = (a.nmma + 31 + kWarps - 1) / kWarps;
    for (int it = 0; it < kAIters; ++it)
        if (m0 + kWarps * it >= 0 && m0 + kWarps * it < kTcRows) a_tile |= 1u << it;
    for (int it = 0; it < b_iters; ++it)
        if (m0 + kWarps * it >= 0 && m0 + kWarps * it < a.nmma) b_tile |= 1u << it;
    const uint32_t a_dst = kmajor_off(m0 + 32, lane) - (32 / 8) * 1024;
    const uint32_t b_dst = a_dst;

    for (int tile = blockIdx.x; tile < a.ntiles && ok; tile += gridDim.x) {
        const int r0 = tile * kTcRows;
        /* A iterations whose row r0 + m0 + kWarps*it is below n */
        uint32_t a_rows = 0;
        for (int it = 0; it < kAIters; ++it)
            if ((long long)r0 + m0 + kWarps * it < a.n) a_rows |= 1u << it;
        /* zero the accumulator: warp w serves lane quarter w%4 */
        {
            const uint32_t q = (uint32_t)(warp & 3);
            for (int c = (warp >> 2) * 32; c < tm_cols; c += 32 * (kWarps / 4)) {
                const uint32_t addr = tmem + ((q * 32) << 16) + (uint32_t)c;
                asm volatile(
                    "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
                    "{%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,"
                    "%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1};"
                    ::"r"(addr), "r"(0u) : "memory");
            }
            asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
        }
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        __syncthreads();
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");

        /* chunk j's operands: cp.async copies straight into the K-major
         * swizzled layout, so no register round trip stalls the warps;
         * kStages chunks in flight.  A cell (m, kk) <- DA[(k0+kk - (r0+m) -
         * a_lo)*n + r0+m]; B cell (nn, kk) <- DB[(nn-kk)*n + k0+kk].  Lane l
         * of walk g covers (g + l, l): one stored diagonal, consecutive rows.
         * Every warp runs the same iterations: a cell outside the tile is
         * skipped by predicate, a cell outside the band is a zero-filled
         * copy (source size 0), so the loops neither diverge nor branch. */
        auto issue = [&](int j) {
            if (j < a.nchunks) {
                const int s = j % kStages;
                const long long k0 = (long long)r0 + a.a_lo + (long long)kTcK * j;
                /* A walk: m = m0 + kWarps*it; per step the diagonal index
                 * ri = k0+lane-r0-m-a_lo = 32j+31-warp-kWarps*it (the same for
                 * the whole warp) shrinks by kWarps, the source moves by
                 * kWarps*(1-n) floats and the destination by kWarps/8
                 * swizzle atoms (kmajor_off is linear in whole atoms). */
                {
                    const int ri0 = kTcK * j + 31 - warp;
                    /* iterations with ri in [0, P) */
                    const int v_lo = ri0 >= a.P ? (ri0 - a.P) / kWarps + 1 : 0;
                    const int v_hi = ri0 >= 0 ? min(ri0 / kWarps + 1, 31) : 0;
                    const uint32_t val = a_rows & (((1u << v_hi) - 1u) & ~((1u << v_lo) - 1u));
                    const uint32_t dst0 = smem_u32(a_stage(s)) + a_dst;
                    const float* src0 = a.DA + (long long)ri0 * a.n + r0 + m0;
                    const long long step = (long long)kWarps * (1 - (long long)a.n);
#pragma unroll
                    for (int it = 0; it < kAIters; ++it) {
                        const bool v = (val >> it) & 1u;
                        cp_async4(dst0 + (uint32_t)(it * (kWarps / 8) * 1024),
                                  v ? src0 + it * step : a.DA, (a_tile >> it) & 1u, v);
                    }
                }
                /* B walk: nn = nn0 + kWarps*it, stored diagonal rj = warp -
                 * 31 + kWarps*it (the same for the whole warp); the source
                 * moves by kWarps*n floats per step. */
                {
                    const long long brow = k0 + lane;
                    const int h0 = warp - 31;
                    const int v_lo = h0 < 0 ? (-h0 + kWarps - 1) / kWarps : 0;
                    const int v_hi = min((a.Q - 1 - h0) / kWarps + 1, 31);
                    const uint32_t val = (brow >= 0 && brow < a.n)
                                             ? ((1u << v_hi) - 1u) & ~((1u << v_lo) - 1u)
                                             : 0u;
                    const uint32_t dst0 = smem_u32(b_stage(s)) + b_dst;
                    const float* src0 = a.DB + (long long)h0 * a.n + brow;
                    const long long step = (long long)kWarps * a.n;
#pragma unroll 6
                    for (int it = 0; it < b_iters; ++it) {
                        const bool v = (val >> it) & 1u;
                        cp_async4(dst0 + (uint32_t)(it * (kWarps / 8) * 1024),
                                  v ? src0 + it * step : a.DB, (b_tile >> it) & 1u, v);
                    }
                }
            }
            asm volatile("cp.async.commit_group;" ::: "memory");
        };
        for (int j = 0; j < kAhead; ++j) issue(j);
        for (int j = 0; j < a.nchunks; ++j) {
            /* refill the stage chunk j-2 used, once its MMAs are done: chunk
             * j-1's MMAs stay in flight while chunk j's copies land, so the
             * MMA latency is not exposed */
            const int sp = (j + kAhead) % kStages;
            if ((pending >> sp) & 1u) {
                if (!mbar_wait(smem_u32(&mbar[sp]), (phase >> sp) & 1u)) ok = false;
                phase ^= 1u << sp;
                pending &= ~(1u << sp);
            }
            if (__syncthreads_or(!ok)) { ok = false; break; }
            issue(j + kAhead);
            asm volatile("cp.async.wait_group %0;" ::"n"(kAhead) : "memory");
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncthreads();
            const int s = j % kStages;
            if (tid == 0) {
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const uint32_t abase = smem_u32(a_stage(s)), bbase = smem_u32(b_stage(s));
                const uint32_t dcol = tmem + (uint32_t)(kTcK * j);
#pragma unroll
                for (int kk = 0; kk < kTcK / 8; ++kk) {
                    const uint64_t ad = smem_desc(abase + 32u * kk);
                    const uint64_t bd = smem_desc(bbase + 32u * kk);
                    asm volatile(
                        "{\n\t.reg .pred p;\n\t"
                        "setp.ne.b32 p, %4, 0;\n\t"
                        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}"
                        ::"r"(dcol), "l"(ad), "l"(bd), "r"(idesc), "r"(1u) : "memory");
                }
                asm volatile(
                    "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                    ::"r"(smem_u32(&mbar[s])) : "memory");
            }
            pending |= 1u << s;
        }
        asm volatile("cp.async.wait_group 0;" ::: "memory");
        /* drain: every committed chunk is waited for exactly once */
        for (int s = 0; s < kStages; ++s)
            if ((pending >> s) & 1u) {
                if (!mbar_wait(smem_u32(&mbar[s]), (phase >> s) & 1u)) ok = false;
                phase ^= 1u << s;
                pending &= ~(1u << s);
            }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        if (__syncthreads_or(!ok)) { ok = false; break; }

        /* epilogue, part 1: accumulator -> shared tile etile[m][t] (TMEM
         * column t of row m is output diagonal kk = t - m).  Warps w and w+4
         * read lane quarter w%4, alternating 32-column windows. */
        {
            const int q = warp & 3;
            float* erow = etile + (32 * q + lane) * kEPitch;
            for (int w = warp >> 2; w * 32 < kECols; w += kWarps / 4) {
                const uint32_t addr = tmem + (((uint32_t)q * 32) << 16) + (uint32_t)(32 * w);
                uint32_t v[32];
                asm volatile(
                    "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
                    "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
                    "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
                    : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]),
                      "=r"(v[6]), "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]),
                      "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]),
                      "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]),
                      "=r"(v[22]), "=r"(v[23]), "=r"(v[24]), "=r"(v[25]), "=r"(v[26]),
                      "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
                    : "r"(addr));
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
                for (int c = 0; c < 32; ++c) erow[32 * w + c] = __uint_as_float(v[c]);
            }
        }
        __syncthreads();
        /* part 2: one warp per output diagonal writes its 128 rows as four
         * coalesced 128-byte runs */
        for (int kk = warp; kk < nk; kk += kWarps) {
            const long long base = kbase[kk];
            const int lo = klo[kk], hi = khi[kk];
#pragma unroll
            for (int i = 0; i < kTcRows / 32; ++i) {
                const int m = 32 * i + lane;
                const long long row = (long long)r0 + m;
                if (row < lo || row >= hi || row >= a.n) continue;
                const float val = etile[m * kEPitch + m + kk];
                float* dst = a.C + base + row;
                if (a.beta)
                    *dst = __fadd_rn(*dst, val);
                else
                    __stcs(dst, val);
            }
        }
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        __syncthreads();
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    }

    if (!ok && tid == 0) atomicOr(&g_device_status, (unsigned)DIA_TC_TIMEOUT);
    /* drain anything still committed before releasing tensor memory */
    for (int s = 0; s < kStages; ++s)
        if ((pending >> s) & 1u) mbar_wait(smem_u32(&mbar[s]), (phase >> s) & 1u);
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 0)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;"
                     ::"r"(tmem), "r"(kTmemCols));
}

/* ===================================================================
 * TMA-fed, warp-specialised variant (the default when the operands meet
 * TMA's alignment rules: n % 4 == 0, 16-byte aligned DA / DB, P, Q <= 256).
 *
 * The 4-byte copies above move one float per lane and cap the bytes an SM
 * keeps in flight; this kernel instead loads whole rectangles of stored
 * diagonals with TMA (cp.async.bulk.tensor.2d, no multicast) into
 * shared-memory rings, and skews them into the MMA operand layout with
 * shared-memory loads and stores:
 *   A row block q of a tile: rows r0+32q .. +31 of all P diagonals
 *     (box 32 x P); a tile has four, and chunk j reads blocks
 *     q in [max(0, (32j-P+1)/32), min(3, j)];
 *   B row block of chunk j: rows k0 .. k0+31 of all Q diagonals, loaded as
 *     36 rows from k0 rounded down to a multiple of 4 (box 36 x Q).
 * Rows outside [0, n) come back as zeros (TMA out-of-bounds fill).
 * Warp roles (26 warps):
 *   warp 0      TMA producer (one thread), in consumption order;
 *   warp 1      MMA issuer (one thread) and tensor-memory owner;
 *   warps 2-9   skew: wait for the raw blocks and a free operand stage,
 *               write the chunk's A and B cells (a cell that a walk of the
 *               previous chunk in the same stage left non-zero and that is
 *               zero now is cleared; B's zero cells never change), release
 *               raw blocks no later chunk needs;
 *   warps 10-25 epilogue: per 32-column window of the 128 x tm
 *               accumulator, tcgen05.ld, release the window to the next
 *               tile's MMAs, then write the window's diagonal runs (<= 32
 *               consecutive rows each) to C.
 * The accumulator is never cleared: the first MMA into a column overwrites
 * it (chunk j writes its last 32 columns first; chunk 0 all of its own).
 * Every hand-off is an mbarrier; every wait gives up after about two
 * seconds, sets DIA_TC_TIMEOUT and makes the other roles stop.
 * =================================================================== */
constexpr int kSkewWarp0 = 2, kSkewWarps = 8;   /* a multiple of 8: walks move by whole atoms */
constexpr int kEpiWarp0 = kSkewWarp0 + kSkewWarps, kEpiWarps = 16;
constexpr int kWsThreads = (kEpiWarp0 + kEpiWarps) * 32;
constexpr int kARing = 4;          /* A row blocks resident: one tile's four */
constexpr int kBRing = 3;          /* B row blocks resident / in flight */
constexpr int kBRows = 36;         /* B box rows: 32 + alignment slack */
constexpr int kWinCols = 32;       /* epilogue window */
constexpr int kMaxWin = kECols / kWinCols;
/* epilogue buffer: element (m, c) at m*33 + 2c, so that both the row-wise
 * writes (lanes = rows) and the diagonal reads (lane l: row base + l,
 * column l; bank stride 35) hit 32 distinct banks */
constexpr int kEbPitch = kWinCols + 1;
constexpr int kEbFloats = kTcRows * kEbPitch + 32;
constexpr unsigned long long kWsWaitNs = 2000000000ull;
/* Limit of every wait of the warp-specialised kernel (kWsWaitNs unless a
 * test lowers it), and a test switch: when set, one skew warp of CTA 0
 * withholds its first operand-ready arrival, so the MMA issuer's wait runs
 * out and the kernel must take its abort path (stop every role, let issued
 * copies land, free tensor memory) and report DIA_TC_TIMEOUT. */
static __device__ unsigned long long g_ws_wait_ns = kWsWaitNs;
static __device__ int g_ws_withhold;

struct WsArgs {
    float* C;
    const int* C_offsets;
    const int* C_lens;
    const int* k_to_idx;
    int n, P, Q, a_lo, b_lo;
    int nchunks, nmma, nwin, ntiles, beta;
    int st_bytes;          /* one operand stage: A slice + B slice */
    int a_slot, b_slot;    /* bytes of one raw A / B block */
    int raw_a_off, raw_b_off, ebuf_off, table_off;
};

struct WsBars {
    unsigned long long full_a[kARing], empty_a[kARing];
    unsigned long long full_b[kBRing], empty_b[kBRing];
    unsigned long long op_full[2], op_empty[2];
    unsigned long long acc_full, drain;
    unsigned long long win_free[kMaxWin];
};

__device__ __forceinline__ unsigned long long global_ns()
{
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity)
{
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

/* Waits for the phase of `bar` with parity `parity`; false if another role
 * aborted or the wait ran past its time limit (then this one aborts). */
__device__ bool ws_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag)
{
    unsigned long long t0 = 0;
    for (int it = 0;; ++it) {
        if (mbar_try(bar, parity)) return true;
        if (*abort_flag) return false;
        /* waiting warps give their issue slots to the working ones */
        __nanosleep(64);
        if ((it & 255) == 0) {
            const unsigned long long t = global_ns();
            if (t0 == 0)
                t0 = t;
            else if (t - t0 > g_ws_wait_ns) {
                *abort_flag = 1;
                atomicOr(&g_device_status, (unsigned)DIA_TC_TIMEOUT);
                return false;
            }
        }
    }
}

/* like ws_wait but ignores the abort flag: used to let copies and MMAs that
 * were already issued finish before the CTA exits */
__device__ void ws_drain(uint32_t bar, uint32_t parity)
{
    const unsigned long long t0 = global_ns();
    while (!mbar_try(bar, parity))
        if (global_ns() - t0 > g_ws_wait_ns) {
            atomicOr(&g_device_status, (unsigned)DIA_TC_TIMEOUT);
            return;
        }
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar)
{
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y,
                                            uint32_t bar, uint32_t bytes)
{
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;"
                 ::"r"(bar), "r"(bytes) : "memory");
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
        "[%0], [%1, {%2, %3}], [%4];"
        ::"r"(dst), "l"((unsigned long long)map), "r"(x), "r"(y), "r"(bar)
        : "memory");
}

__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&v)[8])
{
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]),
                   "=r"(v[6]), "=r"(v[7])
                 : "r"(taddr));
}

/* waits for this thread's tcgen05.ld; the registers are tied in so no use
 * of them can move above the wait */
__device__ __forceinline__ void tmem_wait_ld8(uint32_t (&v)[8])
{
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(v[0]), "+r"(v[1]), "+r"(v[2]), "+r"(v[3]), "+r"(v[4]), "+r"(v[5]),
                   "+r"(v[6]), "+r"(v[7])
                 :
                 : "memory");
}

/* four K = 8 steps of one 32-column chunk: D[dcol..] (+)= A * B; with
 * accumulate false the first step overwrites D */
__device__ __forceinline__ void mma_tf32x4(uint32_t dcol, uint32_t abase, uint32_t bbase,
                                           uint32_t idesc, bool accumulate)
{
#pragma unroll
    for (int kk = 0; kk < kTcK / 8; ++kk) {
        const uint64_t ad = smem_desc(abase + 32u * kk);
        const uint64_t bd = smem_desc(bbase + 32u * kk);
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "setp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}"
            ::"r"(dcol), "l"(ad), "l"(bd), "r"(idesc), "r"((accumulate || kk > 0) ? 1u : 0u)
            : "memory");
    }
}

__device__ __forceinline__ void st_shared(uint32_t addr, float v)
{
    asm volatile("st.shared.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}

__device__ __forceinline__ int floor_div32(int x) { return x >= 0 ? x / 32 : -((31 - x) / 32); }

/* first A row block chunk j reads (nchunks: 4, i.e. all released) */
__device__ __forceinline__ int ws_qlo(int j, int P, int nchunks)
{
    if (j >= nchunks) return 4;
    return max(0, floor_div32(kTcK * j - P + 1));
}

__global__ void __launch_bounds__(kWsThreads, 1)
gemm_diag_ws_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                    WsArgs a)
{
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint32_t sbase = smem_u32(smem);
    const uint32_t raw_a = sbase + a.raw_a_off, raw_b = sbase + a.raw_b_off;
    const float* raw_a_f = (const float*)(smem + a.raw_a_off);
    const float* raw_b_f = (const float*)(smem + a.raw_b_off);
    float* ebuf = (float*)(smem + a.ebuf_off);
    long long* kbase = (long long*)(smem + a.table_off);
    int* klo = (int*)(kbase + kTcMaxDiags);
    int* khi = klo + kTcMaxDiags;
    __shared__ __align__(8) WsBars bars;
    __shared__ uint32_t s_tmem;
    __shared__ int s_abort;
    __shared__ long long s_row_lo, s_row_hi;
    volatile int* abort_flag = &s_abort;
    auto bar = [](unsigned long long& b) { return smem_u32(&b); };

    const int nk = a.P + a.Q - 1;
    for (int kk = tid; kk < nk; kk += kWsThreads) {
        const int k = a.a_lo + a.b_lo + kk;
        const int ki = (k > -a.n && k < a.n) ? a.k_to_idx[k + a.n - 1] : -1;
        if (ki >= 0) {
            const int m = min(k, 0);
            kbase[kk] = (long long)a.C_offsets[ki] + m - kk;   /* minus kk: see the epilogue */
            klo[kk] = -m;
            khi[kk] = a.C_lens[ki] - m;
        } else {
            kbase[kk] = 0;
            klo[kk] = 1;
            khi[kk] = 0;
        }
    }
    __syncthreads();
    if (tid == 0) {
        /* rows [s_row_lo, s_row_hi) lie inside every output diagonal */
        long long lo = 0, hi = a.n;
        for (int kk = 0; kk < nk; ++kk) {
            lo = max(lo, (long long)klo[kk]);
            hi = min(hi, (long long)khi[kk]);
        }
        s_row_lo = lo;
        s_row_hi = hi;
    }
    /* both operand stages start as zeros: B cells outside the band stay
     * zero for good, A cells are cleared where a later chunk needs it */
    for (int i = tid; i < 2 * a.st_bytes / 4; i += kWsThreads) st_shared(sbase + 4 * i, 0.0f);
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    if (tid == 0) {
        s_abort = 0;
        for (int s = 0; s < kARing; ++s) {
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bar(bars.full_a[s])));
            asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;"
                         ::"r"(bar(bars.empty_a[s])), "r"(kSkewWarps));
        }
        for (int s = 0; s < kBRing; ++s) {
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bar(bars.full_b[s])));
            asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;"
                         ::"r"(bar(bars.empty_b[s])), "r"(kSkewWarps));
        }
        for (int s = 0; s < 2; ++s) {
            asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;"
                         ::"r"(bar(bars.op_full[s])), "r"(kSkewWarps));
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bar(bars.op_empty[s])));
        }
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bar(bars.acc_full)));
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bar(bars.drain)));
        for (int w = 0; w < kMaxWin; ++w)
            asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;"
                         ::"r"(bar(bars.win_free[w])), "r"(kEpiWarps));
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     ::"r"(smem_u32(&s_tmem)), "r"(512));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = s_tmem;
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");

    const int a_bytes = kTcRows * kTcK * 4;
    if (warp == 0) {
        /* ---------------- TMA producer */
        if (lane == 0) {
            int ga = 0, gb = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < a.ntiles && ok; tile += gridDim.x) {
                const int r0 = tile * kTcRows;
                for (int j = 0; j < a.nchunks && ok; ++j) {
                    if (j < 4) {
                        const int s = ga % kARing;
                        if (!ws_wait(bar(bars.empty_a[s]), ((ga / kARing) & 1) ^ 1, abort_flag)) {
                            ok = false;
                            break;
                        }
                        tma_load_2d(raw_a + s * a.a_slot, &tmA, r0 + kTcK * j, 0,
                                    bar(bars.full_a[s]), (uint32_t)(kTcK * a.P * 4));
                        ++ga;
                    }
                    const int s = gb % kBRing;
                    if (!ws_wait(bar(bars.empty_b[s]), ((gb / kBRing) & 1) ^ 1, abort_flag)) {
                        ok = false;
                        break;
                    }
                    const int x = r0 + a.a_lo + kTcK * j;
                    tma_load_2d(raw_b + s * a.b_slot, &tmB, x - (x & 3), 0, bar(bars.full_b[s]),
                                (uint32_t)(kBRows * a.Q * 4));
                    ++gb;
                }
            }
            /* no copy may still be landing when the CTA exits */
            for (int i = max(0, ga - kARing); i < ga; ++i)
                ws_drain(bar(bars.full_a[i % kARing]), (i / kARing) & 1);
            for (int i = max(0, gb - kBRing); i < gb; ++i)
                ws_drain(bar(bars.full_b[i % kBRing]), (i / kBRing) & 1);
        }
    } else if (warp == 1) {
        /* ---------------- MMA issuer */
        if (lane == 0) {
            const uint32_t idesc0 = (1u << 4) | (2u << 7) | (2u << 10) |
                                    ((uint32_t)(kTcRows >> 4) << 24);
            int go = 0, u = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < a.ntiles && ok; tile += gridDim.x, ++u) {
                int w_done = 0;
                for (int j = 0; j < a.nchunks; ++j, ++go) {
                    const int w_hi = min(a.nwin, (kTcK * j + a.nmma + kWinCols - 1) / kWinCols);
                    for (; w_done < w_hi && ok; ++w_done)
                        ok = ws_wait(bar(bars.win_free[w_done]), (u & 1) ^ 1, abort_flag);
                    const int s = go & 1;
                    if (!ok || !ws_wait(bar(bars.op_full[s]), (go >> 1) & 1, abort_flag)) {
                        ok = false;
                        break;
                    }
                    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                    const uint32_t abase = sbase + s * a.st_bytes, bbase = abase + a_bytes;
                    /* columns [32j, 32j + nmma - 32) already hold earlier
                     * chunks' sums; the last 32 (all nmma for chunk 0) are
                     * written here first, so their first MMA overwrites and
                     * the accumulator never needs clearing */
                    const int n_old = j == 0 ? 0 : a.nmma - kTcK;
                    const uint32_t dcol = tmem + (uint32_t)(kTcK * j);
                    if (n_old > 0)
                        mma_tf32x4(dcol, abase, bbase, idesc0 | ((uint32_t)(n_old >> 3) << 17), true);
                    mma_tf32x4(dcol + (uint32_t)n_old, abase, bbase + (uint32_t)n_old * 128u,
                               idesc0 | ((uint32_t)((a.nmma - n_old) >> 3) << 17), false);
                    asm volatile(
                        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                        ::"r"(bar(bars.op_empty[s])) : "memory");
                }
                if (ok)
                    asm volatile(
                        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                        ::"r"(bar(bars.acc_full)) : "memory");
            }
            /* every MMA issued has completed before tensor memory is freed */
            asm volatile(
                "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                ::"r"(bar(bars.drain)) : "memory");
            ws_drain(bar(bars.drain), 0);
        }
    } else if (warp < kEpiWarp0) {
        /* ---------------- skew: raw blocks -> swizzled operand stage */
        const int sw = warp - kSkewWarp0;
        int ga0 = 0, gb = 0, go = 0;
        int prev_j[2] = {-1, -1};   /* chunk whose A cells a stage holds (-1: zeros) */
        bool ok = true;
        for (int tile = blockIdx.x; tile < a.ntiles && ok; tile += gridDim.x, ga0 += 4) {
            const int r0 = tile * kTcRows;
            for (int j = 0; j < a.nchunks; ++j, ++go, ++gb) {
                if (j < 4)
                    ok = ws_wait(bar(bars.full_a[(ga0 + j) % kARing]),
                                 ((ga0 + j) / kARing) & 1, abort_flag);
                const int sb = gb % kBRing;
                ok = ok && ws_wait(bar(bars.full_b[sb]), (gb / kBRing) & 1, abort_flag);
                const int s = go & 1;
                ok = ok && ws_wait(bar(bars.op_empty[s]), ((go >> 1) & 1) ^ 1, abort_flag);
                if (!ok) break;
                float* ast = (float*)(smem + s * a.st_bytes);
                float* bst = (float*)(smem + s * a.st_bytes + a_bytes);
                const int jp = s ? prev_j[1] : prev_j[0];
                /* A walks: walk g writes cells (g + l, l) of diagonal d =
                 * 32j - g from raw block m >> 5 (slot = block: a tile's four
                 * blocks fill the ring exactly).  Warps take every kSkewWarps-th
                 * walk, so the swizzled destination moves by whole atoms. */
                const int g_lo = max(-31, kTcK * j - a.P + 1), g_hi = min(kTcRows - 1, kTcK * j);
                {
                    /* four walks per batch: loads first, then stores */
                    const int g0 = g_lo + (((sw - 31 - g_lo) % kSkewWarps) + kSkewWarps) % kSkewWarps;
                    const int nw = g_hi >= g0 ? (g_hi - g0) / kSkewWarps + 1 : 0;
                    const int P32 = a.P * kTcK;
                    for (int i0 = 0; i0 < nw; i0 += 4) {
                        float v[4];
#pragma unroll
                        for (int k = 0; k < 4; ++k) {
                            const int g = g0 + kSkewWarps * (i0 + k);
                            const int m = g + lane;
                            const int d = kTcK * j - g;
                            v[k] = (i0 + k < nw && (unsigned)m < (unsigned)kTcRows)
                                       ? raw_a_f[(m >> 5) * P32 + d * kTcK + (m & 31)]
                                       : 0.0f;
                        }
#pragma unroll
                        for (int k = 0; k < 4; ++k) {
                            const int m = g0 + kSkewWarps * (i0 + k) + lane;
                            if (i0 + k < nw && (unsigned)m < (unsigned)kTcRows)
                                ast[kmajor_off(m, lane) >> 2] = v[k];
                        }
                    }
                }
                /* walks that the stage's previous chunk filled and that are
                 * all zero now */
                if (jp >= 0) {
                    const int p_lo = max(-31, kTcK * jp - a.P + 1), p_hi = min(kTcRows - 1, kTcK * jp);
                    const int g0 = p_lo + (((sw - 31 - p_lo) % kSkewWarps) + kSkewWarps) % kSkewWarps;
                    for (int g = g0; g <= p_hi; g += kSkewWarps) {
                        const int m = g + lane;
                        if ((g < g_lo || g > g_hi) && (unsigned)m < (unsigned)kTcRows)
                            ast[kmajor_off(m, lane) >> 2] = 0.0f;
                    }
                }
                /* B walks: walk b writes cells (b + l, l) of diagonal b; every
                 * b + l < Q + 31 <= nmma lands inside the slice */
                const int x = r0 + a.a_lo + kTcK * j;
                {
                    const float* rb = raw_b_f + sb * (a.b_slot / 4) + (x & 3) + lane + sw * kBRows;
                    float* bd = bst + (kmajor_off(sw + lane, lane) >> 2);
                    const int nw = a.Q > sw ? (a.Q - 1 - sw) / kSkewWarps + 1 : 0;
                    constexpr int kStepSrc = kSkewWarps * kBRows;
                    constexpr int kStepDst = (kSkewWarps / 8) * 256;   /* floats per atom step */
                    for (int i0 = 0; i0 < nw; i0 += 8) {
                        float v[8];
#pragma unroll
                        for (int k = 0; k < 8; ++k)
                            v[k] = i0 + k < nw ? rb[(i0 + k) * kStepSrc] : 0.0f;
#pragma unroll
                        for (int k = 0; k < 8; ++k)
                            if (i0 + k < nw) bd[(i0 + k) * kStepDst] = v[k];
                    }
                }
                if (s) prev_j[1] = j; else prev_j[0] = j;
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                __syncwarp();
                if (lane == 0) {
                    if (!(g_ws_withhold && blockIdx.x == 0 && sw == 0 && go == 0))
                        mbar_arrive(bar(bars.op_full[s]));
                    mbar_arrive(bar(bars.empty_b[sb]));
                    for (int q = ws_qlo(j, a.P, a.nchunks); q < ws_qlo(j + 1, a.P, a.nchunks); ++q)
                        mbar_arrive(bar(bars.empty_a[(ga0 + q) % kARing]));
                }
            }
        }
    } else {
        /* ---------------- epilogue: accumulator windows -> C */
        const int ew = warp - kEpiWarp0;
        const uint32_t q = (uint32_t)(warp & 3);
        const int part = ew >> 2;               /* which 8 of the window's 32 columns */
        const int m_own = 32 * (int)q + lane;
        const uint32_t tlane = tmem + ((q * 32) << 16) + (uint32_t)(8 * part);
        int u = 0;
        bool ok = true;
        for (int tile = blockIdx.x; tile < a.ntiles && ok; tile += gridDim.x, ++u) {
            const long long r0 = (long long)tile * kTcRows;
            if (!ws_wait(bar(bars.acc_full), u & 1, abort_flag)) {
                ok = false;
                break;
            }
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const bool interior = r0 >= s_row_lo && r0 + kTcRows <= s_row_hi && !a.beta;
            uint32_t v[8];
            tmem_ld8(tlane, v);
            tmem_wait_ld8(v);
            for (int w = 0; w < a.nwin; ++w) {
                /* the window is in registers: hand its columns to the next
                 * tile's MMAs, then start reading the next window */
                asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
                __syncwarp();
                if (lane == 0) mbar_arrive(bar(bars.win_free[w]));
                uint32_t vn[8];
                if (w + 1 < a.nwin) tmem_ld8(tlane + (uint32_t)(kWinCols * (w + 1)), vn);
                /* the previous window's runs are written before ebuf is reused */
                asm volatile("bar.sync 1, %0;" ::"n"(kEpiWarps * 32) : "memory");
#pragma unroll
                for (int c = 0; c < 8; ++c)
                    ebuf[m_own * kEbPitch + 2 * (8 * part + c)] = __uint_as_float(v[c]);
                asm volatile("bar.sync 2, %0;" ::"n"(kEpiWarps * 32) : "memory");
                /* window columns t in [T0, T0+32) hold diagonals kk = t - m;
                 * lane l of diagonal kk takes row m = T0 - kk + l, column l */
                const int T0 = kWinCols * w;
                const int kk_lo = max(0, T0 - (kTcRows - 1)), kk_hi = min(nk - 1, T0 + kWinCols - 1);
                if (interior) {
                    /* every row of the tile lies inside every output diagonal */
                    float* crow = a.C + r0 + T0 + lane;
                    const float* eb = ebuf + T0 * kEbPitch + (kEbPitch + 2) * lane;
#pragma unroll 4
                    for (int kk = kk_lo + ew; kk <= kk_hi; kk += kEpiWarps) {
                        if ((unsigned)(T0 - kk + lane) < (unsigned)kTcRows)
                            __stcs(crow + kbase[kk], eb[-kEbPitch * kk]);
                    }
                } else {
                    for (int kk = kk_lo + ew; kk <= kk_hi; kk += kEpiWarps) {
                        const int m = T0 - kk + lane;
                        const long long row = r0 + m;
                        if (m < 0 || m >= kTcRows || row < klo[kk] || row >= khi[kk] || row >= a.n)
                            continue;
                        const float val = ebuf[m * kEbPitch + 2 * lane];
                        float* dst = a.C + kbase[kk] + kk + row;
                        if (a.beta)
                            *dst = __fadd_rn(*dst, val);
                        else
                            __stcs(dst, val);
                    }
                }
                if (w + 1 < a.nwin) {
                    tmem_wait_ld8(vn);
#pragma unroll
                    for (int c = 0; c < 8; ++c) v[c] = vn[c];
                }
            }
        }
    }

    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (warp == 1)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512));
}

static bool contiguous(const int* off, int k)
{
    for (int i = 1; i < k; ++i)
        if (off[i] != off[0] + i) return false;
    return true;
}

/* dynamic shared memory: operand stages overlaid by the epilogue tile, the
 * per-diagonal output table, 1024 bytes of alignment slack */
static int tc_smem_bytes(int nmma)
{
    return std::max(kEpiBytes, kStages * (kTcRows + nmma) * kTcK * 4) +
           kTcMaxDiags * (8 + 4 + 4) + 1024;
}

static int tc_geometry(int P, int Q, int& nchunks, int& nmma)
{
    nchunks = (kTcRows - 1 + P + kTcK - 1) / kTcK;
    nmma = (kTcK - 1 + Q + 15) / 16 * 16;
    return nmma <= 256 && kTcK * (nchunks - 1) + nmma <= kECols &&
           kTcRows - 1 + P + Q - 1 <= kECols && P + Q - 1 <= kTcMaxDiags &&
           tc_smem_bytes(nmma) <= kMaxSmem;
}

int gemm_diag_tc_supported(const int* h_off_A, int P, const int* h_off_B, int Q, int n)
{
    int nc, nm;
    if (P < 1 || Q < 1 || !contiguous(h_off_A, P) || !contiguous(h_off_B, Q))
        return fail(DIA_ERR_UNSUPPORTED,
                    "dia_gemm_diag: tensor-core mode needs contiguous ascending offsets");
    if (!tc_geometry(P, Q, nc, nm))
        return fail(DIA_ERR_UNSUPPORTED, "dia_gemm_diag: band too wide for tensor-core mode "
                                         "(needs P+Q-1 <= 257, a tile accumulator of <= 384 "
                                         "columns and operand stages within shared memory)");
    if (n < 1) return fail(DIA_ERR_UNSUPPORTED, "dia_gemm_diag: empty matrix");
    return DIA_OK;
}

/* cuTensorMapEncodeTiled from the driver, fetched through the runtime so
 * the library needs no link against libcuda */
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_tiled()
{
    static EncodeTiledFn fn = nullptr;
    static bool tried = false;
    if (!tried) {
        tried = true;
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = (EncodeTiledFn)p;
    }
    return fn;
}

/* rows x diags fp32 matrix stored diagonal-major with row stride n; box of
 * box_rows x diags */
static bool make_map(CUtensorMap* map, const float* base, int n, int diags, int box_rows)
{
    EncodeTiledFn fn = encode_tiled();
    if (!fn) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)n, (cuuint64_t)diags};
    const cuuint64_t strides[1] = {(cuuint64_t)n * 4};
    const cuuint32_t box[2] = {(cuuint32_t)box_rows, (cuuint32_t)diags};
    const cuuint32_t estr[2] = {1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, (void*)base, dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

/* shared-memory plan of the warp-specialised kernel; false if it does not
 * fit or TMA cannot address the operands */
static bool ws_plan(const float* DA, const float* DB, int P, int Q, int n, int nmma, WsArgs& w,
                    int& smem)
{
    if (n % 4 != 0 || ((uintptr_t)DA & 15) || ((uintptr_t)DB & 15) || P > 256 || Q > 256)
        return false;
    w.st_bytes = kTcRows * kTcK * 4 + nmma * kTcK * 4;
    w.a_slot = kTcK * P * 4;
    w.b_slot = (kBRows * Q * 4 + 127) / 128 * 128;
    w.raw_a_off = 2 * w.st_bytes;
    w.raw_b_off = w.raw_a_off + kARing * w.a_slot;
    w.ebuf_off = w.raw_b_off + kBRing * w.b_slot;
    w.table_off = w.ebuf_off + kEbFloats * 4;
    smem = w.table_off + kTcMaxDiags * (8 + 4 + 4) + 1024;
    return smem <= kMaxSmem;
}

int gemm_diag_tc_launch(const float* d_DA, const float* d_DB, const int* h_off_A, int P,
                        const int* h_off_B, int Q, int n, float* d_C_data,
                        const int* d_C_offsets, const int* d_C_lens, const int* d_k_to_idx,
                        int beta, cudaStream_t stream)
{
    int nchunks, nmma;
    tc_geometry(P, Q, nchunks, nmma);
    const int ntiles = (n + kTcRows - 1) / kTcRows;
    WsArgs w{};
    int ws_smem = 0;
    CUtensorMap mA, mB;
    if (ws_plan(d_DA, d_DB, P, Q, n, nmma, w, ws_smem) && make_map(&mA, d_DA, n, P, kTcK) &&
        make_map(&mB, d_DB, n, Q, kBRows)) {
        w.C = d_C_data;
        w.C_offsets = d_C_offsets;
        w.C_lens = d_C_lens;
        w.k_to_idx = d_k_to_idx;
        w.n = n;
        w.P = P;
        w.Q = Q;
        w.a_lo = h_off_A[0];
        w.b_lo = h_off_B[0];
        w.nchunks = nchunks;
        w.nmma = nmma;
        w.nwin = (kTcK * (nchunks - 1) + nmma + kWinCols - 1) / kWinCols;
        w.ntiles = ntiles;
        w.beta = beta;
        /* above half of the SM's shared memory: one CTA (the only owner of
         * all 512 TMEM columns) per SM */
        ws_smem = std::max(ws_smem, 120 * 1024);
        DIA_TRY_CUDA(cudaFuncSetAttribute(gemm_diag_ws_kernel,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize, ws_smem));
        const int grid = std::min(ntiles, num_sms());
        gemm_diag_ws_kernel<<<grid, kWsThreads, ws_smem, stream>>>(mA, mB, w);
        DIA_TRY_CUDA(cudaGetLastError());
        return DIA_OK;
    }
    TcArgs a{};
    a.DA = d_DA;
    a.DB = d_DB;
    a.C = d_C_data;
    a.C_offsets = d_C_offsets;
    a.C_lens = d_C_lens;
    a.k_to_idx = d_k_to_idx;
    a.n = n;
    a.P = P;
    a.Q = Q;
    a.a_lo = h_off_A[0];
    a.b_lo = h_off_B[0];
    a.nchunks = nchunks;
    a.nmma = nmma;
    a.ntiles = ntiles;
    a.beta = beta;
    const int smem_need = tc_smem_bytes(a.nmma);
    /* above half of the SM's shared memory: one CTA (one TMEM owner) per SM */
    const int smem = std::max(smem_need, 120 * 1024);
    DIA_TRY_CUDA(cudaFuncSetAttribute(gemm_diag_tc_kernel,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    const int grid = std::min(a.ntiles, num_sms());
    gemm_diag_tc_kernel<<<grid, kTcThreads, smem, stream>>>(a);
    DIA_TRY_CUDA(cudaGetLastError());
    return DIA_OK;
}

}  // namespace dia

extern "C" int dia_device_status(unsigned int* flags, int clear)
{
    if (!flags) return dia::fail(DIA_ERR_INVALID, "dia_device_status: null pointer");
    DIA_TRY_CUDA(cudaMemcpyFromSymbol(flags, dia::g_device_status, sizeof(unsigned int)));
    if (clear) {
        const unsigned int z = 0;
        DIA_TRY_CUDA(cudaMemcpyToSymbol(dia::g_device_status, &z, sizeof(unsigned int)));
    }
    return DIA_OK;
}

extern "C" int dia_test_tc_wait(uint64_t wait_ns, int withhold)
{
    if (wait_ns == 0) wait_ns = dia::kWsWaitNs;
    const unsigned long long ns = wait_ns;
    const int w = withhold ? 1 : 0;
    DIA_TRY_CUDA(cudaMemcpyToSymbol(dia::g_ws_wait_ns, &ns, sizeof(ns)));
    DIA_TRY_CUDA(cudaMemcpyToSymbol(dia::g_ws_withhold, &w, sizeof(w)));
    return DIA_OK;
}
