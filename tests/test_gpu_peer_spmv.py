"""The fused peer-halo SpMV step kernel (dia_spmv_rows_peer) on one GPU.

The kernel's neighbours are emulated with local buffers: before each call
the test puts the neighbours' columns into this rank's receive buffers and
sets the flags, as the neighbours' own kernels would, so the kernel never
has to wait for another launch.  Each emulated rank's rows must equal the
whole-matrix SpMV bit for bit, the columns it pushed must land in the
"peer" buffers, and its flags must carry the step number.  A flag that
nothing sets must make the kernel give up after its time limit, set
DIA_DIST_TIMEOUT and leave the GPU usable.
"""
import ctypes as C

import numpy as np
import pytest
import torch

import diagpu_b200 as dg
import oracle
from diagpu_b200.dist import DIA_DIST_TIMEOUT, Halo, PeerHalo, spmv_rows_peer

pytestmark = pytest.mark.gpu

STENCIL = np.array([i + 64 * j + 4096 * k for k in (-1, 0, 1) for j in (-1, 0, 1)
                    for i in (-1, 0, 1)], np.int32)


class Window:
    """One emulated rank's receive window plus scratch "peer" buffers."""

    def __init__(self, h: Halo):
        rg = h.ranges()
        self.h = h
        self.lo = [torch.full((max(1, h.r0 - h.xlo),), float("nan"), device="cuda")
                   for _ in range(2)]
        self.hi = [torch.full((max(1, h.xhi - h.r1),), float("nan"), device="cuda")
                   for _ in range(2)]
        self.ctl = torch.zeros(8, dtype=torch.int64, device="cuda")   # flags, counters, status
        self.peer_ctl = torch.zeros(2, dtype=torch.int64, device="cuda")
        self.has_left, self.has_right = h.left is not None, h.right is not None
        self.send_left_hi = int(rg[3]) if self.has_left else h.r0
        self.send_right_lo = int(rg[6]) if self.has_right else h.r1
        self.pl = [torch.zeros(max(1, self.send_left_hi - h.r0), device="cuda") for _ in range(2)]
        self.pr = [torch.zeros(max(1, h.r1 - self.send_right_lo), device="cuda")
                   for _ in range(2)]
        s = PeerHalo()
        p = lambda t, off=0: t.data_ptr() + off
        for q in range(2):
            s.halo_lo[q] = p(self.lo[q]) if h.r0 > h.xlo else None
            s.halo_hi[q] = p(self.hi[q]) if h.xhi > h.r1 else None
            s.peer_left_halo_hi[q] = p(self.pl[q]) if self.has_left else None
            s.peer_right_halo_lo[q] = p(self.pr[q]) if self.has_right else None
        s.flag_lo, s.flag_hi = p(self.ctl, 0), p(self.ctl, 8)
        s.push_count, s.status = p(self.ctl, 16), p(self.ctl, 32)
        s.peer_left_flag_hi = p(self.peer_ctl, 8) if self.has_left else None
        s.peer_right_flag_lo = p(self.peer_ctl, 0) if self.has_right else None
        s.send_left_hi, s.send_right_lo = self.send_left_hi, self.send_right_lo
        s.has_left, s.has_right = int(self.has_left), int(self.has_right)
        s.timeout_ns = 2_000_000_000
        self.s = s

    def deliver(self, x, step):
        """What the neighbours' kernels of `step` would have written here."""
        h, q = self.h, step & 1
        if h.r0 > h.xlo:
            self.lo[q][:h.r0 - h.xlo] = x[h.xlo:h.r0]
            self.lo[1 - q].fill_(float("nan"))
        if h.xhi > h.r1:
            self.hi[q][:h.xhi - h.r1] = x[h.r1:h.xhi]
            self.hi[1 - q].fill_(float("nan"))
        if self.has_left:
            self.ctl[0] = step
        if self.has_right:
            self.ctl[1] = step

    def status(self):
        return int(self.ctl[4].item()) & 0xFFFFFFFF


def _run_case(n, offs, world, steps, seed):
    Af = dg.DiaRows.synth(n, n, offs, seed)
    ranks = []
    for r in range(world):
        h = Halo(n, world, r, int(offs.min()), int(offs.max()))
        A = dg.DiaRows.synth(n, n, offs, seed, vrow0=h.r0, nrows=h.r1 - h.r0)
        ranks.append((h, A, Window(h), torch.zeros(A.stride, device="cuda")))
    for step in range(1, steps + 1):
        x = dg.synth_vector(n, seed + 100 * step)
        yf = dg.spmv(Af, x)
        for h, A, w, y in ranks:
            w.deliver(x, step)
            x_own = x[h.r0:h.r1].clone()
            spmv_rows_peer(w.s, step, A, h.r0, h.r1, h.xlo, h.xhi, x_own, y)
            torch.cuda.synchronize()
            assert torch.equal(y[:h.r1 - h.r0], yf[h.r0:h.r1]), (step, h.rank)
            q = step & 1
            if w.has_left:
                assert torch.equal(w.pl[q][:w.send_left_hi - h.r0], x[h.r0:w.send_left_hi])
                assert int(w.peer_ctl[1].item()) == step
            if w.has_right:
                assert torch.equal(w.pr[q][:h.r1 - w.send_right_lo], x[w.send_right_lo:h.r1])
                assert int(w.peer_ctl[0].item()) == step
            assert w.status() == 0
    return Af, ranks


def test_peer_stencil_three_ranks():
    n = 64 * 64 * 96          # 393,216 rows; halo 4,161 columns each side
    _run_case(n, STENCIL, 3, 3, 21)


def test_peer_asymmetric_offsets():
    """Offsets reaching far to one side only; ranks still wait on both
    neighbours (step ordering) and push empty halos where nothing is
    needed."""
    n = 60_000
    offs = np.array([-3, 0, 5, 2000], np.int32)
    _run_case(n, offs, 3, 2, 31)


def test_peer_matches_oracle_small():
    n = 40_000
    offs = np.array([-1500, -1, 0, 1, 1500], np.int32)
    Af, ranks = _run_case(n, offs, 2, 1, 41)
    x = dg.synth_vector(n, 41 + 100)
    ref = oracle.spmv_rowidx(offs, Af.vals.cpu().numpy(), Af.stride, x.cpu().numpy(),
                             ncols=n, nrows=n)
    for h, A, w, y in ranks:
        assert np.array_equal(y[:h.r1 - h.r0].cpu().numpy(), ref[h.r0:h.r1])


def test_peer_wait_times_out_and_recovers():
    """A flag nothing sets: the boundary tiles give up after 1 ms, the status
    says so, and the next step (flags delivered) is exact again."""
    n = 64 * 64 * 96
    world, rank = 3, 1
    h = Halo(n, world, rank, int(STENCIL.min()), int(STENCIL.max()))
    A = dg.DiaRows.synth(n, n, STENCIL, 51, vrow0=h.r0, nrows=h.r1 - h.r0)
    Af = dg.DiaRows.synth(n, n, STENCIL, 51)
    w = Window(h)
    w.s.timeout_ns = 1_000_000
    y = torch.zeros(A.stride, device="cuda")
    x = dg.synth_vector(n, 52)
    x_own = x[h.r0:h.r1].clone()
    spmv_rows_peer(w.s, 1, A, h.r0, h.r1, h.xlo, h.xhi, x_own, y)   # flags stay 0
    torch.cuda.synchronize()
    assert w.status() & DIA_DIST_TIMEOUT
    w.ctl[4] = 0
    w.s.timeout_ns = 2_000_000_000
    w.deliver(x, 2)
    spmv_rows_peer(w.s, 2, A, h.r0, h.r1, h.xlo, h.xhi, x_own, y)
    torch.cuda.synchronize()
    assert w.status() == 0
    assert torch.equal(y[:h.r1 - h.r0], dg.spmv(Af, x)[h.r0:h.r1])


def test_peer_rejects_bad_arguments():
    n = 64 * 64 * 96
    h = Halo(n, 3, 1, int(STENCIL.min()), int(STENCIL.max()))
    A = dg.DiaRows.synth(n, n, STENCIL, 1, vrow0=h.r0, nrows=h.r1 - h.r0)
    w = Window(h)
    x_own = torch.zeros(h.r1 - h.r0, device="cuda")
    y = torch.zeros(A.stride, device="cuda")
    with pytest.raises(dg.DiaError):
        spmv_rows_peer(w.s, 0, A, h.r0, h.r1, h.xlo, h.xhi, x_own, y)     # steps count from 1
    w.s.has_left = 0
    with pytest.raises(dg.DiaError):                                       # halo without neighbour
        spmv_rows_peer(w.s, 1, A, h.r0, h.r1, h.xlo, h.xhi, x_own, y)
