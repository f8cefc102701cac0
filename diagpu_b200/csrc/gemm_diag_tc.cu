/*
 * gemm_diag_tc.cu -- tcgen05 TF32 dense-band kernel for gemm_diag.
 *
 * When A and B are contiguous bands (offsets a_lo..a_lo+P-1, b_lo..b_lo+Q-1),
 * a tile of 128 consecutive rows of C = A*B is a dense product
 *     C[r0:r0+128, cols] = A[r0:r0+128, K] * B[K, cols]
 * over the K = 127+P columns the tile's A rows touch.  The kernel:
 *   - splits K into 32-column chunks; for chunk j it builds, in shared
 *     memory, the dense 128x32 slice of A and the (31+Q, padded to 16)x32
 *     slice of B in the K-major 128-byte-swizzled layout the tensor core
 *     reads (one 128-byte row per operand row, 8-row atoms).  Each warp walks one
 *     stored diagonal per instruction, so every global load is a coalesced
 *     run of consecutive rows; the tensor core reads the fp32 bits as TF32
 *     (low 13 mantissa bits ignored);
 *   - one thread issues four tcgen05.mma.kind::tf32 (K = 8 each) per chunk,
 *     accumulating into a 128 x 384 fp32 tile in tensor memory (zeroed
 *     first), chunk j landing at TMEM column 32*j; chunks are double
 *     buffered and tcgen05.commit -> mbarrier tells the builders when a
 *     buffer is free again;
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

#include "../../include/diagpu_b200.h"
#include "dia_core.cuh"

namespace dia {

constexpr int kTcRows = 128;        /* M of the MMA: rows per tile */
constexpr int kTcK = 32;            /* columns per K-chunk */
constexpr int kTcThreads = 512;
constexpr int kWarps = kTcThreads / 32;
constexpr int kStages = 5;           /* K-chunks in flight */
constexpr int kTcMaxDiags = 257;    /* P + Q - 1 */
constexpr int kECols = 384;         /* accumulator columns copied out */
constexpr int kEPitch = kECols + 1; /* odd pitch: conflict-free rows and diagonals */
constexpr int kEpiBytes = kTcRows * kEPitch * 4;
constexpr uint32_t kTmemCols = 512;
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
    long long* kbase = (long long*)(smem + kEpiBytes);
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
    uint32_t phase[kStages] = {};
    int pending[kStages] = {};
    bool ok = true;

    for (int tile = blockIdx.x; tile < a.ntiles && ok; tile += gridDim.x) {
        const int r0 = tile * kTcRows;
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
         * core-matrix layout (4 bytes each, zero-filled outside the band), so
         * no register round trip stalls the warps; kStages chunks in flight.
         * A cell (m, kk) <- DA[(k0+kk - (r0+m) - a_lo)*n + r0+m]; B cell
         * (nn, kk) <- DB[(nn-kk)*n + k0+kk].  Lane l of walk g covers
         * (g + l, l): one stored diagonal, consecutive rows. */
        auto issue = [&](int j) {
            if (j < a.nchunks) {
                const int s = j % kStages;
                const long long k0 = (long long)r0 + a.a_lo + (long long)kTcK * j;
                /* A walk: m = g + lane with g = warp - 31 + kWarps*it; per step
                 * m grows by kWarps, the diagonal index ri = k0+lane-r0-m-a_lo
                 * shrinks by kWarps, so the source moves by kWarps*(1-n)
                 * floats and the destination by kWarps/8 core-matrix rows. */
                {
                    const int m0 = warp - 31 + lane;             /* m at it = 0 */
                    const long long ri0 = k0 + lane - r0 - m0 - a.a_lo;
                    /* iterations with m in [0, 128) */
                    int it_lo = m0 < 0 ? (-m0 + kWarps - 1) / kWarps : 0;
                    int it_hi = m0 < kTcRows ? (kTcRows - 1 - m0) / kWarps + 1 : 0;
                    /* iterations with ri in [0, P) and row < n */
                    long long v_lo = ri0 >= a.P ? (ri0 - a.P) / kWarps + 1 : 0;
                    long long v_hi = ri0 >= 0 ? ri0 / kWarps + 1 : 0;
                    const long long rows_left = (long long)a.n - r0 - m0;   /* row < n */
                    const long long n_hi = rows_left > 0 ? (rows_left - 1) / kWarps + 1 : 0;
                    v_hi = v_hi < n_hi ? v_hi : n_hi;
                    uint32_t dst = smem_u32(a_stage(s)) + kmajor_off(m0 + kWarps * it_lo, lane);
                    const int va = (int)(v_lo > it_lo ? (v_lo < it_hi ? v_lo : it_hi) : it_lo);
                    const int vb = (int)(v_hi > va ? (v_hi < it_hi ? v_hi : it_hi) : va);
                    int it = it_lo;
                    for (; it < va; ++it, dst += 128 * kWarps)
                        asm volatile("st.shared.f32 [%0], %1;" ::"r"(dst), "f"(0.0f) : "memory");
                    if (it < vb) {
                        const float* src = a.DA + (ri0 - (long long)kWarps * it) * a.n +
                                           (r0 + m0 + kWarps * it);
                        const long long step = (long long)kWarps * (1 - (long long)a.n);
                        for (; it < vb; ++it, dst += 128 * kWarps, src += step)
                            asm volatile("cp.async.ca.shared.global [%0], [%1], 4;"
                                         ::"r"(dst), "l"(src) : "memory");
                    }
                    for (; it < it_hi; ++it, dst += 128 * kWarps)
                        asm volatile("st.shared.f32 [%0], %1;" ::"r"(dst), "f"(0.0f) : "memory");
                }
                /* B walk: nn = h + lane, rj = h = warp - 31 + kWarps*it; the
                 * source moves by kWarps*n floats per step. */
                {
                    const long long brow = k0 + lane;
                    const bool brow_ok = brow >= 0 && brow < a.n;
                    const int nn0 = warp - 31 + lane;
                    const int h0 = warp - 31;
                    int it_lo = nn0 < 0 ? (-nn0 + kWarps - 1) / kWarps : 0;
                    int it_hi = nn0 < a.nmma ? (a.nmma - 1 - nn0) / kWarps + 1 : 0;
                    const int v_lo = h0 < 0 ? (-h0 + kWarps - 1) / kWarps : 0;
                    const int v_hi = brow_ok ? (h0 < a.Q ? (a.Q - 1 - h0) / kWarps + 1 : 0) : 0;
                    uint32_t dst = smem_u32(b_stage(s)) + kmajor_off(nn0 + kWarps * it_lo, lane);
                    const int va = v_lo > it_lo ? (v_lo < it_hi ? v_lo : it_hi) : it_lo;
                    const int vb = v_hi > va ? (v_hi < it_hi ? v_hi : it_hi) : va;
                    int it = it_lo;
                    for (; it < va; ++it, dst += 128 * kWarps)
                        asm volatile("st.shared.f32 [%0], %1;" ::"r"(dst), "f"(0.0f) : "memory");
                    if (it < vb) {
                        const float* src = a.DB + (long long)(h0 + kWarps * it) * a.n + brow;
                        const long long step = (long long)kWarps * a.n;
                        for (; it < vb; ++it, dst += 128 * kWarps, src += step)
                            asm volatile("cp.async.ca.shared.global [%0], [%1], 4;"
                                         ::"r"(dst), "l"(src) : "memory");
                    }
                    for (; it < it_hi; ++it, dst += 128 * kWarps)
                        asm volatile("st.shared.f32 [%0], %1;" ::"r"(dst), "f"(0.0f) : "memory");
                }
            }
            asm volatile("cp.async.commit_group;" ::: "memory");
        };
        for (int j = 0; j < kStages - 1; ++j) issue(j);
        for (int j = 0; j < a.nchunks; ++j) {
            /* refill the stage chunk j-1 used, once its MMAs are done */
            const int sp = (j + kStages - 1) % kStages;
            if (pending[sp]) {
                if (!mbar_wait(smem_u32(&mbar[sp]), phase[sp])) ok = false;
                phase[sp] ^= 1u;
                pending[sp] = 0;
            }
            if (__syncthreads_or(!ok)) { ok = false; break; }
            issue(j + kStages - 1);
            asm volatile("cp.async.wait_group %0;" ::"n"(kStages - 1) : "memory");
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
            pending[s] = 1;
        }
        asm volatile("cp.async.wait_group 0;" ::: "memory");
        /* drain: every committed chunk is waited for exactly once */
        for (int s = 0; s < kStages; ++s)
            if (pending[s]) {
                if (!mbar_wait(smem_u32(&mbar[s]), phase[s])) ok = false;
                phase[s] ^= 1u;
                pending[s] = 0;
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
        if (pending[s]) mbar_wait(smem_u32(&mbar[s]), phase[s]);
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 0)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;"
                     ::"r"(tmem), "r"(kTmemCols));
}

static bool contiguous(const int* off, int k)
{
    for (int i = 1; i < k; ++i)
        if (off[i] != off[0] + i) return false;
    return true;
}

static int tc_geometry(int P, int Q, int& nchunks, int& nmma)
{
    nchunks = (kTcRows - 1 + P + kTcK - 1) / kTcK;
    nmma = (kTcK - 1 + Q + 15) / 16 * 16;
    return nmma <= 256 && kTcK * (nchunks - 1) + nmma <= kECols &&
           kTcRows - 1 + P + Q - 1 <= kECols && P + Q - 1 <= kTcMaxDiags &&
           kStages * (kTcRows + nmma) * kTcK * 4 <= kEpiBytes;
}

int gemm_diag_tc_supported(const int* h_off_A, int P, const int* h_off_B, int Q, int n)
{
    int nc, nm;
    if (P < 1 || Q < 1 || !contiguous(h_off_A, P) || !contiguous(h_off_B, Q))
        return fail(DIA_ERR_UNSUPPORTED,
                    "dia_gemm_diag: tensor-core mode needs contiguous ascending offsets");
    if (!tc_geometry(P, Q, nc, nm))
        return fail(DIA_ERR_UNSUPPORTED, "dia_gemm_diag: band too wide for tensor-core mode "
                                         "(needs P+Q-1 <= 257)");
    if (n < 1) return fail(DIA_ERR_UNSUPPORTED, "dia_gemm_diag: empty matrix");
    return DIA_OK;
}

int gemm_diag_tc_launch(const float* d_DA, const float* d_DB, const int* h_off_A, int P,
                        const int* h_off_B, int Q, int n, float* d_C_data,
                        const int* d_C_offsets, const int* d_C_lens, const int* d_k_to_idx,
                        int beta, cudaStream_t stream)
{
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
    tc_geometry(P, Q, a.nchunks, a.nmma);
    a.ntiles = (n + kTcRows - 1) / kTcRows;
    a.beta = beta;
    const int smem_need = kEpiBytes + kTcMaxDiags * (8 + 4 + 4) + 1024;
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
