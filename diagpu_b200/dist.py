"""Row-block partitioning and halo exchange across GPUs.

A matrix of order n is split into contiguous row blocks, one per rank
(a multiple of 32 rows each, so every block starts 128-byte aligned in the
padded rows layout).  Row i of y = A*x needs x columns i + d for every
offset d, so rank r, owning rows [r0, r1), needs x on [r0 + min d, r1 + max d):
its own columns plus a halo of max|d| columns from each neighbour.  For
C = A*B the same holds for the rows of B (halo = max|d_A|).  The halo is the
only communication: NCCL point-to-point sends/receives with ranks r-1 and
r+1 (batched), issued before the interior rows' kernel so the transfer over
NVLink overlaps the interior compute; the boundary rows run after the
receive completes.  The reference has no multi-GPU path; this module is the
partitioned form of its single-GPU products.

The exchange is written against torch.distributed and works with the nccl
backend (GPU tensors) and gloo (CPU tensors, used by the CPU tests).
"""
from __future__ import annotations

import numpy as np
import torch
import torch.distributed as dist

from . import DiaRows, SpmspmPlan, spmspm_symbolic, spmv


def row_block(n: int, world: int, rank: int, align: int = 32):
    """[r0, r1) of rank's rows: equal shares rounded to `align` rows."""
    per = -(-n // world)
    per = -(-per // align) * align
    r0 = min(n, rank * per)
    r1 = min(n, r0 + per)
    return r0, r1


def halo_window(n: int, r0: int, r1: int, lo_off: int, hi_off: int):
    """Global columns [xlo, xhi) rows [r0, r1) touch for offsets in
    [lo_off, hi_off] (clipped to the matrix)."""
    return max(0, r0 + min(lo_off, 0)), min(n, r1 + max(hi_off, 0))


class Halo:
    """Halo geometry of one rank for offsets in [lo_off, hi_off]."""

    def __init__(self, n, world, rank, lo_off, hi_off):
        self.n, self.world, self.rank = n, world, rank
        self.lo_off, self.hi_off = min(lo_off, 0), max(hi_off, 0)
        self.r0, self.r1 = row_block(n, world, rank)
        self.xlo, self.xhi = halo_window(n, self.r0, self.r1, self.lo_off, self.hi_off)
        for r in range(world):
            a, b = row_block(n, world, r)
            if 0 < b - a < max(-self.lo_off, self.hi_off) and world > 1:
                raise ValueError(f"halo {max(-self.lo_off, self.hi_off)} exceeds rank {r}'s "
                                 f"{b - a} rows: use fewer ranks")
        # what each neighbour needs from me
        self.left = row_block(n, world, rank - 1) if rank > 0 else None
        self.right = row_block(n, world, rank + 1) if rank < world - 1 else None

    @property
    def width(self):
        return self.xhi - self.xlo

    def interior(self):
        """Rows whose columns all lie in this rank's own [r0, r1)."""
        a = self.r0 - self.lo_off if self.rank > 0 else self.r0
        b = self.r1 - self.hi_off if self.rank < self.world - 1 else self.r1
        a, b = min(max(a, self.r0), self.r1), max(min(b, self.r1), self.r0)
        return (a, max(a, b))

    def boundary(self):
        a, b = self.interior()
        return [(lo, hi) for lo, hi in ((self.r0, a), (b, self.r1)) if hi > lo]

    def ranges(self):
        """Global column ranges [recv-left, send-left, recv-right, send-right]
        as 8 int64 (the exchange start() posts; empty where no neighbour)."""
        r = [0] * 8
        if self.left is not None:
            lxlo, lxhi = halo_window(self.n, *self.left, self.lo_off, self.hi_off)
            r[0:4] = [self.xlo, self.r0, self.r0, max(self.r0, lxhi)]
        if self.right is not None:
            rxlo, rxhi = halo_window(self.n, *self.right, self.lo_off, self.hi_off)
            r[4:8] = [self.r1, self.xhi, min(rxlo, self.r1), self.r1]
        return np.array(r, np.int64)

    def start(self, ext: torch.Tensor, group=None):
        """Post the halo sends/receives on ext (column j = global xlo + j);
        returns a handle whose wait() completes the exchange."""
        e2 = ext.view(1, -1) if ext.dim() == 1 else ext
        ops, post = [], []

        def cols(a, b):
            return e2[:, a - self.xlo:b - self.xlo]

        def recv(a, b, peer):
            v = cols(a, b)
            buf = v if v.is_contiguous() else torch.empty(v.shape, dtype=v.dtype, device=v.device)
            ops.append(dist.P2POp(dist.irecv, buf, peer, group))
            if buf is not v:
                post.append((v, buf))

        def send(a, b, peer):
            v = cols(a, b)
            buf = v if v.is_contiguous() else v.contiguous()
            ops.append(dist.P2POp(dist.isend, buf, peer, group))

        if self.left is not None:
            lxlo, lxhi = halo_window(self.n, *self.left, self.lo_off, self.hi_off)
            if self.xlo < self.r0:
                recv(self.xlo, self.r0, self.rank - 1)
            if lxhi > self.r0:
                send(self.r0, lxhi, self.rank - 1)
        if self.right is not None:
            rxlo, rxhi = halo_window(self.n, *self.right, self.lo_off, self.hi_off)
            if self.xhi > self.r1:
                recv(self.r1, self.xhi, self.rank + 1)
            if rxlo < self.r1:
                send(rxlo, self.r1, self.rank + 1)
        works = dist.batch_isend_irecv(ops) if ops else []
        return _Pending(works, post)


class _NativeWait:
    def __init__(self, comm):
        self.comm = comm

    def wait(self):
        from . import _stream, check, lib
        check(lib().dia_dist_halo_wait(self.comm.handle, _stream()))


class _Pending:
    def __init__(self, works, post):
        self.works, self.post = works, post

    def wait(self, timeout=None):
        """Complete the exchange; with `timeout` (a datetime.timedelta) a
        neighbour that never posts its side raises instead of blocking."""
        for w in self.works:
            if timeout is None:
                w.wait()
            else:
                w.wait(timeout)
        for v, buf in self.post:
            v.copy_(buf)


class NativeComm:
    """The library's own NCCL communicator and halo stream (dia_dist_*),
    created collectively from a unique id broadcast over torch.distributed.
    Used by DistSpmv / DistSpmspm when the process group runs NCCL."""

    def __init__(self, group=None):
        import ctypes as C
        from . import check, lib
        rank, world = dist.get_rank(group), dist.get_world_size(group)
        idbuf = bytearray(128)
        if rank == 0:
            cbuf = (C.c_char * 128)()
            check(lib().dia_nccl_unique_id(cbuf, 128))
            idbuf = bytearray(cbuf.raw)
        obj = [bytes(idbuf)]
        dist.broadcast_object_list(obj, src=0, group=group)
        raw = (C.c_char * 128).from_buffer_copy(obj[0])
        self._h = C.c_void_p()
        check(lib().dia_dist_create(rank, world, raw, C.byref(self._h)))
        self.rank, self.world = rank, world

    @property
    def handle(self):
        return self._h

    def check(self):
        from . import check, lib
        check(lib().dia_dist_async_error(self._h))

    def peer_setup(self, halo: "Halo"):
        """Map the neighbours' receive windows (collective); afterwards
        dia_dist_spmv_fused moves the x halo inside the step kernel."""
        from . import check, lib
        self._ranges = halo.ranges()
        check(lib().dia_dist_peer_setup(self._h, halo.r0, halo.r1, halo.xlo, halo.xhi,
                                        self._ranges.ctypes.data))

    def set_timeout(self, seconds: float):
        from . import check, lib
        check(lib().dia_dist_set_timeout(self._h, int(seconds * 1e9)))

    def status(self, clear=True) -> int:
        """DIA_DIST_* bits the step kernels set (DIA_DIST_TIMEOUT = 2)."""
        import ctypes as C
        from . import check, lib
        v = C.c_uint(0)
        check(lib().dia_dist_status(self._h, C.byref(v), int(clear)))
        return v.value

    def __del__(self):
        from . import _lib
        if getattr(self, "_h", None) and self._h.value and _lib is not None:
            _lib.dia_dist_destroy(self._h)
            self._h = None


def use_native(group=None):
    return dist.is_initialized() and dist.get_backend(group) == "nccl"


# ----------------------------------------------------------------- products

DIA_DIST_TIMEOUT = 2
PEER = 3


def _peer_halo_struct():
    import ctypes as C
    fp, u64p = C.c_void_p, C.c_void_p

    class PeerHalo(C.Structure):
        """Mirror of DiaPeerHalo (include/diagpu_b200.h): device pointers of
        this rank's receive window and of the neighbours' windows."""
        _fields_ = [("halo_lo", fp * 2), ("halo_hi", fp * 2), ("flag_lo", u64p),
                    ("flag_hi", u64p), ("push_count", u64p), ("status", fp),
                    ("peer_left_halo_hi", fp * 2), ("peer_left_flag_hi", u64p),
                    ("peer_right_halo_lo", fp * 2), ("peer_right_flag_lo", u64p),
                    ("send_left_hi", C.c_int64), ("send_right_lo", C.c_int64),
                    ("has_left", C.c_int), ("has_right", C.c_int), ("timeout_ns", C.c_int64)]
    return PeerHalo


PeerHalo = _peer_halo_struct()


def spmv_rows_peer(halo: "PeerHalo", step, A: DiaRows, r0, r1, xlo, xhi, x_own, y, stream=None):
    """One fused peer-halo SpMV step with explicit buffers
    (dia_spmv_rows_peer); y row i is written at y[i - A.vrow0]."""
    import ctypes as C
    from . import _dptr, _stream, check, lib
    offs = np.asarray(A.offsets)
    check(lib().dia_spmv_rows_peer(C.byref(halo), step, A.n_rows, A.n_cols, A.K,
                                   _dptr(A.d_offsets), _dptr(A.vals), A.stride, A.vrow0, r0, r1,
                                   xlo, xhi, int(offs.min()), int(offs.max()),
                                   _dptr(x_own, torch.float32), _dptr(y, torch.float32),
                                   _stream(stream)))
    return y


class DistSpmv:
    """y = A*x with A row-partitioned over the process group.

    Each rank holds its row block of A (padded rows layout) and an extended
    x buffer over its halo window.  With NCCL, `step()` is one library call.
    overlap=3 (PEER, the default): one fused kernel per step moves the halo
    over NVLink itself (dia_dist_spmv_fused; peer windows mapped once at
    construction).  The NCCL forms (dia_dist_spmv_step): 2, halo and
    boundary strips on the library's high-priority stream concurrently with
    the interior rows; 1, boundary strips after the interior on one stream;
    0, exchange, then one launch over the block.  Without NCCL (gloo/CPU
    groups) the exchange goes through torch.distributed."""

    def __init__(self, A: DiaRows, halo: Halo, group=None, native=None, overlap=PEER):
        self.A, self.halo, self.group = A, halo, group
        dev = A.vals.device
        self.x_ext = torch.zeros(halo.width, dtype=torch.float32, device=dev)
        self.y = torch.zeros(A.stride, dtype=torch.float32, device=dev)
        if native is None and halo.world > 1 and use_native(group):
            native = NativeComm(group)
        self.native = native
        self.overlap = overlap
        self._ranges = halo.ranges()
        if self.native is not None and overlap == PEER:
            if not getattr(self.native, "_peer", False):
                self.native.peer_setup(halo)
                self.native._peer = True
        offs = np.asarray(A.offsets)
        self._dmin, self._dmax = int(offs.min()), int(offs.max())

    @property
    def x_own(self):
        h = self.halo
        return self.x_ext[h.r0 - h.xlo:h.r1 - h.xlo]

    def step(self, launches: list | None = None):
        h = self.halo
        if self.native is not None:
            return self._native_step(launches)
        pend = h.start(self.x_ext, self.group) if h.world > 1 else None
        a, b = h.interior()
        if b > a:
            spmv(self.A, self.x_ext, self.y, x_lo=h.xlo, row_lo=a, row_hi=b)
            if launches is not None:
                launches.append("spmv")
        if pend is not None:
            pend.wait()
        for lo, hi in h.boundary():
            spmv(self.A, self.x_ext, self.y, x_lo=h.xlo, row_lo=lo, row_hi=hi)
            if launches is not None:
                launches.append("spmv")
        return self.y


    def _native_step(self, launches):
        import ctypes as C
        from . import _dptr, _stream, check, lib
        h, A = self.halo, self.A
        if self.overlap == PEER:
            check(lib().dia_dist_spmv_fused(self.native.handle, A.n_rows, A.n_cols, A.K,
                                            _dptr(A.d_offsets), _dptr(A.vals), A.stride,
                                            A.vrow0, self._dmin, self._dmax, _dptr(self.x_own),
                                            _dptr(self.y), _stream()))
            if launches is not None:
                launches.append("peer_spmv")
            return self.y
        a, b = h.interior()
        check(lib().dia_dist_spmv_step(self.native.handle, A.n_rows, A.n_cols, A.K,
                                       _dptr(A.d_offsets), _dptr(A.vals), A.stride, A.vrow0,
                                       _dptr(self.x_ext), h.xlo, h.xhi, _dptr(self.y),
                                       self._ranges.ctypes.data_as(C.c_void_p), h.r0, h.r1,
                                       a, b, int(self.overlap), _stream()))
        if launches is not None:
            launches += (["spmv"] * (int(b > a) + int(a > h.r0) + int(h.r1 > b))
                         if self.overlap else ["spmv"])
        if self.overlap == 2 and h.world > 1:
            pass  # the boundary strips ran on the library's halo stream
        return self.y


class DistSpmspm:
    """C = A*B with A, B, C row-partitioned; B's halo rows (within max|d_A|
    of the block) come from the neighbours.  Two plans: one whose B range is
    this rank's own rows (interior rows, run while the halo is in flight)
    and one over the whole halo window (boundary rows, run after it)."""

    def __init__(self, A: DiaRows, B_ext: DiaRows, halo: Halo, group=None):
        self.A, self.B, self.halo, self.group = A, B_ext, halo, group
        h = halo
        self.plan_own = SpmspmPlan(A, B_ext, b_lo=h.r0, b_hi=h.r1)
        self.plan_all = SpmspmPlan(A, B_ext, b_lo=h.xlo, b_hi=h.xhi)
        self.C = self.plan_all.new_C()
        self.sym = spmspm_symbolic(A.n_rows, A.offsets, B_ext.offsets)
        self.native = NativeComm(group) if halo.world > 1 and use_native(group) else None
        self._ranges = halo.ranges()

    def step(self, launches: list | None = None):
        h = self.halo
        if self.native is not None:
            import ctypes as C
            from . import _dptr, _stream, check, lib
            B = self.B
            check(lib().dia_dist_halo_start(self.native.handle, _dptr(B.vals), B.vrow0, B.stride,
                                            B.K, self._ranges.ctypes.data_as(C.c_void_p),
                                            _stream()))
            pend = _NativeWait(self.native)
        else:
            pend = h.start(self.B.vals, self.group) if h.world > 1 else None
        a, b = h.interior()
        plan_in = self.plan_all if pend is None else self.plan_own
        if b > a:
            plan_in.execute(self.A, self.B, self.C, a, b)
            if launches is not None:
                launches += ["tile_sum", "pair_sum"]
        if pend is not None:
            pend.wait()
        for lo, hi in h.boundary():
            self.plan_all.execute(self.A, self.B, self.C, lo, hi)
            if launches is not None:
                launches += ["pair_sum"]
        return self.C


def offsets_span(offsets):
    o = np.asarray(offsets)
    return int(o.min()), int(o.max())


class PeerLost(RuntimeError):
    """A neighbour stopped taking part (left, or missed its heartbeat)."""


class Heartbeat:
    """Host-side liveness of the ranks of a partitioned product.

    Before each step a rank publishes the step it is about to run in the
    process group's key-value store and waits, at most `timeout` seconds,
    until both neighbours have published the same step (every rank
    publishes before it waits, so the handshake cannot deadlock).  A rank
    that leaves between steps (calls leave(), or simply stops) is therefore
    noticed by its neighbours on the host, before they launch a step kernel
    that would wait for it or write into its freed receive window.  The
    check costs a few store round trips per step, so it is for runs that
    need failure detection, not for the timed loop."""

    def __init__(self, halo: Halo, store=None, prefix="dia_hb", timeout=5.0):
        import torch.distributed.distributed_c10d as c10d
        self.halo = halo
        self.store = store if store is not None else c10d._get_default_store()
        self.prefix, self.timeout = prefix, float(timeout)
        self.step = 0
        self.neighbours = [r for r in (halo.rank - 1, halo.rank + 1) if 0 <= r < halo.world]

    def _key(self, r):
        return f"{self.prefix}/{r}"

    def beat(self):
        """Announce the next step and wait (bounded) for the neighbours to
        announce it too; raises PeerLost otherwise."""
        import time
        self.step += 1
        self.store.set(self._key(self.halo.rank), str(self.step))
        deadline = time.monotonic() + self.timeout
        for r in self.neighbours:
            while True:
                v = self._read(r)
                if v == "left":
                    raise PeerLost(f"rank {r} left before step {self.step}")
                if v is not None and int(v) >= self.step:
                    break
                if time.monotonic() > deadline:
                    raise PeerLost(f"rank {r} missed its heartbeat for step {self.step}")
                time.sleep(0.01)

    def _read(self, r):
        import datetime
        try:
            self.store.wait([self._key(r)], datetime.timedelta(milliseconds=50))
        except Exception:  # noqa: BLE001 - key not there yet
            return None
        return self.store.get(self._key(r)).decode()

    def leave(self):
        """Tell the neighbours this rank takes part in no further step."""
        self.store.set(self._key(self.halo.rank), "left")
