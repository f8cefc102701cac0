/*
 * dist.cu -- native NCCL halo exchange for row-partitioned products.
 *
 * One process per GPU; each rank owns a contiguous row block.  Before a
 * product, a rank needs the columns (x entries, or B rows) within the
 * largest offset of its block boundaries from its two neighbours.  This
 * file owns an NCCL communicator (created from a unique id the caller
 * distributes once, e.g. through torch.distributed) and a private stream:
 *   halo_start: the private stream waits for the caller's stream, then one
 *               ncclGroupStart/End posts every send/receive with ranks r-1
 *               and r+1 (one pair per stored row of the exchanged buffer);
 *   halo_wait:  the caller's stream waits for the exchange.
 * dia_dist_spmv_step enqueues a whole partitioned SpMV with one host call.
 * In its default mode the halo stream has the highest priority: NCCL's
 * transfer and then the two boundary strips run there, concurrently with
 * the interior rows' kernel (local columns only) on the caller's stream,
 * and their CTAs are dispatched ahead of the interior kernel's pending
 * ones.  The driver's 8-GPU run of this form (config 5) measured 0.218
 * ms per step against 0.172 ms for the block's kernel alone; the exchange
 * and the strips, not the kernel, were the cost, which is why the default
 * step is now the fused peer-halo kernel of dist_peer.cu.
 * The reference has no multi-GPU path (its programs run on one device).
 */
#include <nccl.h>

#include <chrono>
#include <cstring>
#include <string>
#include <thread>
#include <vector>

#include "../../include/diagpu_b200.h"
#include "dia_core.cuh"

struct DiaDist {
    ncclComm_t comm = nullptr;
    cudaStream_t cs = nullptr;
    cudaEvent_t ready = nullptr, done = nullptr;
    int rank = 0, world = 1;
    /* peer-memory halo (dia_dist_peer_setup) */
    void* window = nullptr;        /* this rank's receive window */
    void* peer_win[2] = {nullptr, nullptr}; /* IPC mappings of left / right windows */
    DiaPeerHalo ph{};
    uint64_t step = 0;
    int64_t r0 = 0, r1 = 0, x_lo = 0, x_hi = 0;
    bool peer_ready = false;
    int64_t comm_timeout_ms = 120000;   /* deadline of each host-side NCCL completion */
};

namespace {

int nccl_fail(ncclResult_t r, const char* what)
{
    return dia::fail(DIA_ERR_CUDA, std::string(what) + ": " + ncclGetErrorString(r));
}

#define DIA_TRY_NCCL(expr)                                  \
    do {                                                    \
        ncclResult_t r__ = (expr);                          \
        if (r__ != ncclSuccess) return nccl_fail(r__, #expr); \
    } while (0)

/* The communicator is non-blocking: a call may return ncclInProgress while
 * NCCL finishes it in the background (connection set-up, init bootstrap).
 * Completion is polled here against a deadline; a communicator that does
 * not complete in time (a rank that never joined, a peer that stopped
 * answering during set-up) is aborted and the call returns DIA_ERR_TIMEOUT,
 * instead of the process blocking forever.  Only host-side completion is
 * covered: a transfer that the GPU has started waits on the GPU, which is
 * why ranks check each other on the host before every step. */
int nccl_complete(DiaDist* d, ncclResult_t r, const char* what)
{
    if (r == ncclSuccess) return DIA_OK;
    if (r != ncclInProgress) return nccl_fail(r, what);
    const auto t0 = std::chrono::steady_clock::now();
    for (;;) {
        ncclResult_t st = ncclSuccess;
        const ncclResult_t q = ncclCommGetAsyncError(d->comm, &st);
        if (q != ncclSuccess) return nccl_fail(q, what);
        if (st == ncclSuccess) return DIA_OK;
        if (st != ncclInProgress) return nccl_fail(st, what);
        const auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(
                            std::chrono::steady_clock::now() - t0).count();
        if (ms > d->comm_timeout_ms) {
            ncclCommAbort(d->comm);
            d->comm = nullptr;
            return dia::fail(DIA_ERR_TIMEOUT, std::string(what) + ": not complete after " +
                                             std::to_string(d->comm_timeout_ms) +
                                             " ms; communicator aborted");
        }
        std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
}

#define DIA_NCCL_DONE(d, expr)                                      \
    do {                                                            \
        const int rc__ = nccl_complete((d), (expr), #expr);          \
        if (rc__ != DIA_OK) return rc__;                            \
    } while (0)

int need_comm(const DiaDist* d, const char* who)
{
    if (!d) return dia::fail(DIA_ERR_INVALID, std::string(who) + ": null handle");
    if (!d->comm) return dia::fail(DIA_ERR_INVALID, std::string(who) + ": communicator was aborted");
    return DIA_OK;
}

/* ranges: recv-left [0,1), send-left [2,3), recv-right [4,5), send-right
 * [6,7) as global column indices; ext column j holds global column
 * ext_lo + j, stored rows k*pitch apart. */
int halo_post(DiaDist* d, float* ext, int64_t ext_lo, int64_t pitch, int K,
              const int64_t* rg)
{
    DIA_TRY_NCCL(ncclGroupStart());
    for (int k = 0; k < K; ++k) {
        float* row = ext + (int64_t)k * pitch - ext_lo;
        const int peer[4] = {d->rank - 1, d->rank - 1, d->rank + 1, d->rank + 1};
        for (int s = 0; s < 4; ++s) {
            const int64_t lo = rg[2 * s], hi = rg[2 * s + 1];
            if (hi <= lo || peer[s] < 0 || peer[s] >= d->world) continue;
            if (s % 2 == 0)
                DIA_TRY_NCCL(ncclRecv(row + lo, (size_t)(hi - lo), ncclFloat, peer[s], d->comm,
                                      d->cs));
            else
                DIA_TRY_NCCL(ncclSend(row + lo, (size_t)(hi - lo), ncclFloat, peer[s], d->comm,
                                      d->cs));
        }
    }
    DIA_NCCL_DONE(d, ncclGroupEnd());
    return DIA_OK;
}

}  // namespace

using namespace dia;

extern "C" int dia_nccl_unique_id(void* out, int nbytes)
{
    if (!out || nbytes < (int)sizeof(ncclUniqueId))
        return fail(DIA_ERR_INVALID, "dia_nccl_unique_id: buffer smaller than ncclUniqueId");
    ncclUniqueId id;
    DIA_TRY_NCCL(ncclGetUniqueId(&id));
    std::memcpy(out, &id, sizeof(id));
    return DIA_OK;
}

extern "C" int dia_dist_create_timeout(int rank, int world, const void* id, int64_t timeout_ms,
                                       DiaDist** out)
{
    if (!out || !id || world < 1 || rank < 0 || rank >= world || timeout_ms <= 0)
        return fail(DIA_ERR_INVALID, "dia_dist_create: bad rank/world/timeout or null pointer");
    *out = nullptr;
    auto* d = new DiaDist();
    d->rank = rank;
    d->world = world;
    d->comm_timeout_ms = timeout_ms;
    ncclUniqueId uid;
    std::memcpy(&uid, id, sizeof(uid));
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 0;
    const int rc0 = nccl_complete(d, ncclCommInitRankConfig(&d->comm, world, uid, rank, &cfg),
                                  "ncclCommInitRankConfig");
    if (rc0 != DIA_OK) {
        if (d->comm) ncclCommAbort(d->comm);
        delete d;
        return rc0;
    }
    /* the halo stream gets the highest priority: its small kernels (NCCL's,
     * the boundary strips) are then dispatched ahead of the interior
     * kernel's pending CTAs instead of after them */
    int lo_prio = 0, hi_prio = 0;
    cudaDeviceGetStreamPriorityRange(&lo_prio, &hi_prio);
    cudaError_t e = cudaStreamCreateWithPriority(&d->cs, cudaStreamNonBlocking, hi_prio);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&d->ready, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&d->done, cudaEventDisableTiming);
    if (e != cudaSuccess) {
        ncclCommAbort(d->comm);
        delete d;
        return cuda_fail(e, "dia_dist_create stream/events");
    }
    *out = d;
    return DIA_OK;
}

extern "C" int dia_dist_create(int rank, int world, const void* id, DiaDist** out)
{
    return dia_dist_create_timeout(rank, world, id, 120000, out);
}

extern "C" int dia_dist_abort(DiaDist* d)
{
    if (!d) return fail(DIA_ERR_INVALID, "dia_dist_abort: null handle");
    if (d->comm) ncclCommAbort(d->comm);
    d->comm = nullptr;
    return DIA_OK;
}

extern "C" int dia_dist_halo_start(DiaDist* d, float* d_ext, int64_t ext_lo, int64_t pitch, int K,
                                   const int64_t* h_ranges, cudaStream_t stream)
{
    if (!d || !d_ext || !h_ranges || K < 0)
        return fail(DIA_ERR_INVALID, "dia_dist_halo_start: null pointer or bad K");
    if (int rc = need_comm(d, "dia_dist_halo_start")) return rc;
    DIA_TRY_CUDA(cudaEventRecord(d->ready, stream));
    DIA_TRY_CUDA(cudaStreamWaitEvent(d->cs, d->ready, 0));
    const int rc = halo_post(d, d_ext, ext_lo, pitch, K, h_ranges);
    if (rc) return rc;
    DIA_TRY_CUDA(cudaEventRecord(d->done, d->cs));
    return DIA_OK;
}

extern "C" int dia_dist_halo_wait(DiaDist* d, cudaStream_t stream)
{
    if (!d) return fail(DIA_ERR_INVALID, "dia_dist_halo_wait: null handle");
    DIA_TRY_CUDA(cudaStreamWaitEvent(stream, d->done, 0));
    return DIA_OK;
}

extern "C" int dia_dist_spmv_step(DiaDist* d, int64_t n_rows, int64_t n_cols, int K,
                                  const int* d_offsets, const float* d_vals, int64_t stride,
                                  int64_t vrow0, float* d_x_ext, int64_t x_lo, int64_t x_hi,
                                  float* d_y, const int64_t* h_ranges, int64_t r0, int64_t r1,
                                  int64_t int_lo, int64_t int_hi, int overlap,
                                  cudaStream_t stream)
{
    if (int rc0 = need_comm(d, "dia_dist_spmv_step")) return rc0;
    int rc = DIA_OK;
    if (!overlap) {
        /* exchange first, then one launch over the whole block: the halo is
         * a few hundred KB (tens of microseconds over NVLink), while two
         * extra boundary launches cost their tail latency each */
        if (d->world > 1) {
            rc = dia_dist_halo_start(d, d_x_ext, x_lo, 0, 1, h_ranges, stream);
            if (rc == DIA_OK) rc = dia_dist_halo_wait(d, stream);
            if (rc) return rc;
        }
        return dia_spmv_rows(n_rows, n_cols, K, d_offsets, d_vals, stride, vrow0, r0, r1, d_x_ext,
                             x_lo, x_hi, d_y, stream);
    }
    if (overlap == 2 && d->world > 1) {
        /* the boundary strips run on the halo stream right after the
         * receive, concurrently with the interior rows on `stream`; `stream`
         * then waits for them (they write disjoint rows of y) */
        DIA_TRY_CUDA(cudaEventRecord(d->ready, stream));
        DIA_TRY_CUDA(cudaStreamWaitEvent(d->cs, d->ready, 0));
        rc = halo_post(d, d_x_ext, x_lo, 0, 1, h_ranges);
        if (rc == DIA_OK && int_lo > r0)
            rc = dia_spmv_rows(n_rows, n_cols, K, d_offsets, d_vals, stride, vrow0, r0, int_lo,
                               d_x_ext, x_lo, x_hi, d_y, d->cs);
        if (rc == DIA_OK && r1 > int_hi)
            rc = dia_spmv_rows(n_rows, n_cols, K, d_offsets, d_vals, stride, vrow0, int_hi, r1,
                               d_x_ext, x_lo, x_hi, d_y, d->cs);
        if (rc) return rc;
        DIA_TRY_CUDA(cudaEventRecord(d->done, d->cs));
        if (int_hi > int_lo)
            rc = dia_spmv_rows(n_rows, n_cols, K, d_offsets, d_vals, stride, vrow0, int_lo,
                               int_hi, d_x_ext, x_lo, x_hi, d_y, stream);
        if (rc) return rc;
        return dia_dist_halo_wait(d, stream);
    }
    if (d->world > 1) {
        rc = dia_dist_halo_start(d, d_x_ext, x_lo, 0, 1, h_ranges, stream);
        if (rc) return rc;
    }
    if (int_hi > int_lo)
        rc = dia_spmv_rows(n_rows, n_cols, K, d_offsets, d_vals, stride, vrow0, int_lo, int_hi,
                           d_x_ext, x_lo, x_hi, d_y, stream);
    if (rc) return rc;
    if (d->world > 1) {
        rc = dia_dist_halo_wait(d, stream);
        if (rc) return rc;
    }
    if (int_lo > r0)
        rc = dia_spmv_rows(n_rows, n_cols, K, d_offsets, d_vals, stride, vrow0, r0, int_lo,
                           d_x_ext, x_lo, x_hi, d_y, stream);
    if (rc == DIA_OK && r1 > int_hi)
        rc = dia_spmv_rows(n_rows, n_cols, K, d_offsets, d_vals, stride, vrow0, int_hi, r1,
                           d_x_ext, x_lo, x_hi, d_y, stream);
    return rc;
}

extern "C" int dia_dist_async_error(DiaDist* d)
{
    if (int rc = need_comm(d, "dia_dist_async_error")) return rc;
    ncclResult_t ar = ncclSuccess;
    DIA_TRY_NCCL(ncclCommGetAsyncError(d->comm, &ar));
    if (ar != ncclSuccess && ar != ncclInProgress) return nccl_fail(ar, "NCCL async error");
    return DIA_OK;
}

extern "C" int dia_dist_destroy(DiaDist* d)
{
    if (!d) return DIA_OK;
    if (d->cs) cudaStreamSynchronize(d->cs);
    if (d->window) {
        /* every step kernel of this rank has finished, and each of them
         * waited for both neighbours' last pushes into this window */
        cudaDeviceSynchronize();
        for (void* p : d->peer_win)
            if (p) cudaIpcCloseMemHandle(p);
        cudaFree(d->window);
    }
    if (d->comm) {
        /* non-blocking: finalize completes in the background, then destroy */
        if (nccl_complete(d, ncclCommFinalize(d->comm), "ncclCommFinalize") == DIA_OK && d->comm)
            ncclCommDestroy(d->comm);
        else if (d->comm)
            ncclCommAbort(d->comm);
    }
    if (d->ready) cudaEventDestroy(d->ready);
    if (d->done) cudaEventDestroy(d->done);
    if (d->cs) cudaStreamDestroy(d->cs);
    delete d;
    return DIA_OK;
}

/* ------------------------------------------------------ peer-memory halo */

namespace {

/* Receive window layout: a 256-byte control block (flag_lo, flag_hi,
 * push_count[2], status), then halo_lo[2] and halo_hi[2], each rounded up to
 * 64 floats. */
struct WinLayout {
    size_t lo_off[2], hi_off[2], bytes;
};

WinLayout win_layout(int64_t lo_len, int64_t hi_len)
{
    auto r64 = [](int64_t v) { return (size_t)((v + 63) / 64 * 64) * sizeof(float); };
    WinLayout w{};
    size_t o = 256;
    for (int p = 0; p < 2; ++p) { w.lo_off[p] = o; o += r64(lo_len); }
    for (int p = 0; p < 2; ++p) { w.hi_off[p] = o; o += r64(hi_len); }
    w.bytes = o;
    return w;
}

struct PeerInfo {
    cudaIpcMemHandle_t handle;
    int64_t lo_len, hi_len;
    int64_t valid;
};

}  // namespace

extern "C" int dia_dist_peer_setup(DiaDist* d, int64_t r0, int64_t r1, int64_t x_lo, int64_t x_hi,
                                   const int64_t* rg)
{
    if (!d || !rg) return fail(DIA_ERR_INVALID, "dia_dist_peer_setup: null pointer");
    if (int rc = need_comm(d, "dia_dist_peer_setup")) return rc;
    if (d->window) return fail(DIA_ERR_INVALID, "dia_dist_peer_setup: already set up");
    if (x_lo > r0 || x_hi < r1 || r1 < r0)
        return fail(DIA_ERR_INVALID, "dia_dist_peer_setup: inconsistent halo window");
    const int64_t lo_len = r0 - x_lo, hi_len = x_hi - r1;
    const WinLayout w = win_layout(lo_len, hi_len);
    DIA_TRY_CUDA(cudaMalloc(&d->window, w.bytes));
    DIA_TRY_CUDA(cudaMemset(d->window, 0, w.bytes));
    PeerInfo mine{};
    cudaError_t e = cudaIpcGetMemHandle(&mine.handle, d->window);
    mine.valid = e == cudaSuccess;
    mine.lo_len = lo_len;
    mine.hi_len = hi_len;
    /* every rank takes part in the exchange even when its handle failed, so
     * that all ranks see the failure instead of hanging in the collective */
    PeerInfo* dbuf = nullptr;
    DIA_TRY_CUDA(cudaMalloc(&dbuf, sizeof(PeerInfo) * (size_t)(d->world + 1)));
    DIA_TRY_CUDA(cudaMemcpy(dbuf + d->world, &mine, sizeof(mine), cudaMemcpyHostToDevice));
    const int grc = nccl_complete(d, ncclAllGather(dbuf + d->world, dbuf, sizeof(PeerInfo),
                                                   ncclChar, d->comm, d->cs),
                                  "dia_dist_peer_setup: ncclAllGather");
    const ncclResult_t nr = grc == DIA_OK ? ncclSuccess : ncclInternalError;
    std::vector<PeerInfo> all((size_t)d->world);
    if (nr == ncclSuccess) e = cudaStreamSynchronize(d->cs);
    if (nr == ncclSuccess && e == cudaSuccess)
        e = cudaMemcpy(all.data(), dbuf, sizeof(PeerInfo) * (size_t)d->world,
                       cudaMemcpyDeviceToHost);
    cudaFree(dbuf);
    if (grc != DIA_OK) return grc;
    if (e != cudaSuccess) return cuda_fail(e, "dia_dist_peer_setup: handle exchange");
    for (const PeerInfo& pi : all)
        if (!pi.valid)
            return fail(DIA_ERR_UNSUPPORTED,
                        "dia_dist_peer_setup: cudaIpcGetMemHandle failed on some rank");
    DiaPeerHalo& h = d->ph;
    h = DiaPeerHalo{};
    char* base = (char*)d->window;
    auto* ctl = (unsigned long long*)base;
    h.flag_lo = ctl + 0;
    h.flag_hi = ctl + 1;
    h.push_count = ctl + 2;
    h.status = (unsigned int*)(ctl + 4);
    for (int p = 0; p < 2; ++p) {
        h.halo_lo[p] = lo_len ? (float*)(base + w.lo_off[p]) : nullptr;
        h.halo_hi[p] = hi_len ? (float*)(base + w.hi_off[p]) : nullptr;
    }
    h.timeout_ns = 2000000000LL;
    h.send_left_hi = r0;
    h.send_right_lo = r1;
    for (int side = 0; side < 2; ++side) {
        const int peer = side == 0 ? d->rank - 1 : d->rank + 1;
        if (peer < 0 || peer >= d->world) continue;
        const PeerInfo& pi = all[(size_t)peer];
        /* what this rank sends must be what the neighbour expects */
        const int64_t send = side == 0 ? rg[3] - r0 : r1 - rg[6];
        const int64_t want = side == 0 ? pi.hi_len : pi.lo_len;
        if (send != want || send < 0)
            return fail(DIA_ERR_INVALID, "dia_dist_peer_setup: halo lengths disagree with the "
                                         "neighbour's window");
        void* pw = nullptr;
        DIA_TRY_CUDA(cudaIpcOpenMemHandle(&pw, pi.handle, cudaIpcMemLazyEnablePeerAccess));
        d->peer_win[side] = pw;
        const WinLayout pwl = win_layout(pi.lo_len, pi.hi_len);
        auto* pctl = (unsigned long long*)pw;
        if (side == 0) {
            h.has_left = 1;
            h.peer_left_flag_hi = pctl + 1;
            for (int p = 0; p < 2; ++p) h.peer_left_halo_hi[p] = (float*)((char*)pw + pwl.hi_off[p]);
            h.send_left_hi = rg[3] > r0 ? rg[3] : r0;
        } else {
            h.has_right = 1;
            h.peer_right_flag_lo = pctl + 0;
            for (int p = 0; p < 2; ++p) h.peer_right_halo_lo[p] = (float*)((char*)pw + pwl.lo_off[p]);
            h.send_right_lo = rg[6] < r1 ? rg[6] : r1;
        }
    }
    d->r0 = r0;
    d->r1 = r1;
    d->x_lo = x_lo;
    d->x_hi = x_hi;
    d->step = 0;
    /* no rank may push into a window before its owner has zeroed it */
    DIA_TRY_CUDA(cudaDeviceSynchronize());
    int* one = nullptr;
    DIA_TRY_CUDA(cudaMalloc(&one, sizeof(int)));
    const int brc = nccl_complete(d, ncclAllReduce(one, one, 1, ncclInt, ncclSum, d->comm, d->cs),
                                  "dia_dist_peer_setup: barrier");
    if (brc == DIA_OK) e = cudaStreamSynchronize(d->cs);
    cudaFree(one);
    if (brc != DIA_OK) return brc;
    if (e != cudaSuccess) return cuda_fail(e, "dia_dist_peer_setup: barrier");
    d->peer_ready = true;
    return DIA_OK;
}

extern "C" int dia_dist_spmv_fused(DiaDist* d, int64_t n_rows, int64_t n_cols, int K,
                                   const int* d_offsets, const float* d_vals, int64_t stride,
                                   int64_t vrow0, int dmin, int dmax, const float* d_x_own,
                                   float* d_y, cudaStream_t stream)
{
    if (!d || !d->peer_ready)
        return fail(DIA_ERR_INVALID, "dia_dist_spmv_fused: call dia_dist_peer_setup first");
    const int rc = dia_spmv_rows_peer(&d->ph, d->step + 1, n_rows, n_cols, K, d_offsets, d_vals,
                                      stride, vrow0, d->r0, d->r1, d->x_lo, d->x_hi, dmin, dmax,
                                      d_x_own, d_y, stream);
    if (rc == DIA_OK) ++d->step;
    return rc;
}

extern "C" int dia_dist_set_timeout(DiaDist* d, int64_t ns)
{
    if (!d || ns <= 0) return fail(DIA_ERR_INVALID, "dia_dist_set_timeout: bad argument");
    d->ph.timeout_ns = ns;
    return DIA_OK;
}

extern "C" int dia_dist_status(DiaDist* d, unsigned int* flags, int clear)
{
    if (!d || !flags) return fail(DIA_ERR_INVALID, "dia_dist_status: null pointer");
    *flags = 0;
    if (!d->window) return DIA_OK;
    DIA_TRY_CUDA(cudaMemcpy(flags, d->ph.status, sizeof(unsigned int), cudaMemcpyDeviceToHost));
    if (clear) DIA_TRY_CUDA(cudaMemset(d->ph.status, 0, sizeof(unsigned int)));
    return DIA_OK;
}
