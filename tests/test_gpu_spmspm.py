"""SpMSpM parity on the GPU against cpu_dia_spgemm (golden outputs of the
compiled reference, and the oracle restatement at full config sizes).
FP32 in the reference's summation order: equality is required."""
import numpy as np
import pytest
import torch

import diagpu_b200 as dg
import oracle
from tests._util import dev, hm_to_rows, rel_l2, rows_to_hm, same

pytestmark = pytest.mark.gpu


def _hm(g, name, tag):
    return tuple(g[f"{name}__{tag}_{f}"] for f in ("off", "len", "start", "val"))


def _n(A):
    return int(A[1][A[0] == 0][0])


def _lookup(n, off):
    lk = np.full(2 * n - 1, -1, np.int32)
    for i, d in enumerate(off):
        lk[d + n - 1] = i
    return lk


def run_hm(n, A, B, Cs):
    Co, Cl, Cst = Cs
    nnz = int(Cst[-1] + Cl[-1]) if len(Cl) else 0
    Cv = torch.full((max(nnz, 1),), np.nan, device="cuda")
    dg.spmspm_hm(dev(A[3]), dev(A[2]), dev(A[0]), dev(A[1]), dev(B[3]), dev(B[2]), dev(B[1]),
                 dev(_lookup(n, B[0])), Cv, dev(Cst), dev(Co), dev(Cl), n)
    return Cv.cpu().numpy()[:nnz]


@pytest.mark.parametrize("fixture", ["spmspm_banded", "spmspm_scatter"])
def test_golden_hm(golden, fixture):
    g = golden[fixture]
    for name in g["names"]:
        A, B = _hm(g, name, "A"), _hm(g, name, "B")
        n = _n(A)
        Cs = (g[f"{name}__C_off"], g[f"{name}__C_len"], g[f"{name}__C_start"])
        got = run_hm(n, A, B, Cs)
        assert same(got, g[f"{name}__C_val"]), name


@pytest.mark.parametrize("fixture", ["spmspm_banded", "spmspm_scatter"])
def test_golden_rows_layout(golden, fixture):
    g = golden[fixture]
    for name in g["names"]:
        A, B = _hm(g, name, "A"), _hm(g, name, "B")
        n = _n(A)
        dA = dg.DiaRows.from_host(n, n, A[0], hm_to_rows(n, *A)[:, :n])
        dB = dg.DiaRows.from_host(n, n, B[0], hm_to_rows(n, *B)[:, :n])
        Cm = dg.spmspm(dA, dB)
        assert np.array_equal(Cm.offsets, g[f"{name}__C_off"])
        rows = Cm.vals.cpu().numpy()
        ln, st, val = rows_to_hm(n, Cm.offsets, rows)
        assert same(val, g[f"{name}__C_val"]), name
        # padding mask: every entry outside the matrix is exactly zero
        for k, d in enumerate(Cm.offsets):
            r0 = -min(d, 0)
            mask = np.ones(Cm.stride, bool)
            mask[r0:r0 + ln[k]] = False
            assert (rows[k, mask] == 0).all()


def _rows_product(n, offsA, offsB, seedA, seedB, kind=0):
    A = dg.DiaRows.synth(n, n, offsA, seed=seedA, kind=kind, lo=-1.0 if kind == 0 else 0.0,
                         hi=1.0)
    B = A if offsB is None else dg.DiaRows.synth(n, n, offsB, seed=seedB, kind=kind,
                                                  lo=-1.0 if kind == 0 else 0.0, hi=1.0)
    Cm = dg.spmspm(A, B)
    return A, B, Cm


def _oracle_from_rows(n, A, B, Cm):
    a = rows_to_hm(n, A.offsets, A.vals.cpu().numpy())
    b = rows_to_hm(n, B.offsets, B.vals.cpu().numpy())
    off, ln, st = oracle.c_structure(n, A.offsets, B.offsets)
    ref = oracle.dia_spgemm_hm(n, (A.offsets, *a), (B.offsets, *b), (off, ln, st))
    got = rows_to_hm(n, Cm.offsets, Cm.vals.cpu().numpy())[2]
    return got, ref, (off, ln, st), a, b


def test_config2_stencil_full():
    """Config 2: 3D 7-point stencil on 128^3, C = A*A, 25 output diagonals."""
    n = 128 ** 3
    offs = np.array([-16384, -128, -1, 0, 1, 128, 16384], np.int32)
    A, B, Cm = _rows_product(n, offs, None, 201, None)
    assert Cm.K == 25
    got, ref, *_ = _oracle_from_rows(n, A, B, Cm)
    assert same(got, ref)


def _scatter_offsets(seed):
    rng = np.random.default_rng(seed)
    s = {0}
    while len(s) < 32:
        s.add(int(rng.integers(-512, 513)))
    return np.array(sorted(s), np.int32)


def test_config3_scattered_full():
    """Config 3: n = 1e6, 32 + 32 scattered offsets, normal values."""
    n = 1_000_000
    A, B, Cm = _rows_product(n, _scatter_offsets(301), _scatter_offsets(302), 303, 304, kind=1)
    got, ref, (off, ln, st), a, b = _oracle_from_rows(n, A, B, Cm)
    assert same(got, ref)
    ref64 = oracle.dia_spgemm_hm(n, (A.offsets, *a), (B.offsets, *b), (off, ln, st), f64=True)
    assert rel_l2(got, ref64) <= 1e-6


def test_hm_matches_rows_on_config3_shape():
    n = 200_000
    A, B, Cm = _rows_product(n, _scatter_offsets(7), _scatter_offsets(8), 9, 10)
    a = rows_to_hm(n, A.offsets, A.vals.cpu().numpy())
    b = rows_to_hm(n, B.offsets, B.vals.cpu().numpy())
    off, ln, st = oracle.c_structure(n, A.offsets, B.offsets)
    got = run_hm(n, (A.offsets, *a), (B.offsets, *b), (off, ln, st))
    assert same(got, rows_to_hm(n, Cm.offsets, Cm.vals.cpu().numpy())[2])


def test_config5_windows():
    """Config 5 C = A*A (n = 67M, 125 output diagonals, 33.5 GB of C) at
    full size; checked on row windows against the oracle."""
    n = 256 * 256 * 1024
    offs = np.array([i + 256 * j + 65536 * k for k in (-1, 0, 1) for j in (-1, 0, 1)
                     for i in (-1, 0, 1)], np.int32)
    A = dg.DiaRows.synth(n, n, offs, seed=601)
    Cm = dg.spmspm(A, A)
    assert Cm.K == 125
    H = 65793
    for lo in (0, n // 3 + 5, n - 4096):
        hi = min(n, lo + 4096)
        wlo, whi = max(0, lo - H), min(n, hi + H)
        W = oracle.synth_rowidx(601, n, n, offs, row0=wlo, nrows=whi - wlo)
        Aw = dg.DiaRows.from_host(n, n, offs, W[:, :whi - wlo], vrow0=wlo)
        Cw = dg.DiaRows.empty(n, n, Cm.offsets, vrow0=lo, nrows=hi - lo)
        Aa = dg.DiaRows.from_host(n, n, offs, W[:, lo - wlo:hi - wlo], vrow0=lo)
        dg.spmspm(Aa, Aw, Cw)
        assert same(Cm.vals[:, lo:hi].cpu().numpy(), Cw.vals[:, :hi - lo].cpu().numpy()), lo
        # and the window product against the oracle, exactly
        win_n_ref = _window_oracle(n, offs, W, wlo, lo, hi, Cm.offsets)
        assert same(Cw.vals[:, :hi - lo].cpu().numpy(), win_n_ref), lo
    del Cm


def _window_oracle(n, offs, W, wlo, lo, hi, C_off):
    """C rows [lo, hi) by the HM oracle on the sub-problem (CPU), written
    out in rows layout."""
    out = np.zeros((len(C_off), hi - lo), np.float32)
    Ad = {int(d): k for k, d in enumerate(offs)}
    for c, dc in enumerate(C_off):
        acc = np.zeros(hi - lo, np.float32)
        rows = np.arange(lo, hi)
        valid_c = (rows + dc >= 0) & (rows + dc < n)
        for a, da in enumerate(offs):
            db = int(dc) - int(da)
            if db not in Ad:
                continue
            b = Ad[db]
            r = rows + da
            ok = valid_c & (rows + da >= 0) & (rows + da < n)
            av = W[a, rows - wlo]
            bv = np.zeros(hi - lo, np.float32)
            bv[ok] = W[b, r[ok] - wlo]
            prod = np.where(ok, av * bv, np.float32(0))
            acc = np.where(ok, acc + prod, acc).astype(np.float32)
        out[c] = np.where(valid_c, acc, 0)
    return out


def _runs(starts, P):
    return np.array([s + u for s in starts for u in range(P)], np.int32)


# runs of 3, 4 and 5 whose starts fall on different residues mod 8, so the
# run-pair kernel meets many alignment shifts of its B windows
RUN_CASES = {
    "runs3": (150_001, _runs([-2824, -2181, 409, 1558, 2261], 3)),
    "runs4": (120_003, _runs([-1478, -572, 2155, 2928], 4)),
    "runs5": (90_001, _runs([457, 1102, 1159, 2491], 5)),
}


@pytest.mark.parametrize("case", ["stencil7", "stencil27", "runs2", "band", "scatter", "tiny",
                                  *RUN_CASES])
def test_tiled_plan_equals_generic(case):
    """The shared-memory-tiled path, the planned generic path and the
    unplanned entry point give identical results (and the tiled kernel is
    actually used where the offsets allow it)."""
    if case == "stencil7":
        n, offs = 64 ** 3, np.array([-4096, -64, -1, 0, 1, 64, 4096], np.int32)
    elif case == "stencil27":
        n = 64 * 64 * 64
        offs = np.array([i + 64 * j + 4096 * k for k in (-1, 0, 1) for j in (-1, 0, 1)
                         for i in (-1, 0, 1)], np.int32)
    elif case == "runs2":     # runs of two, asymmetric, odd n
        n, offs = 200_001, np.array([-3001, -3000, -8, -7, 40, 41, 9000, 9001], np.int32)
    elif case == "band":
        n, offs = 100_003, np.arange(-9, 10, dtype=np.int32)
    elif case == "scatter":
        n, offs = 300_000, _scatter_offsets(5)
    elif case in RUN_CASES:
        n, offs = RUN_CASES[case]
    else:
        n, offs = 300, np.array([-2, 0, 1], np.int32)
    A = dg.DiaRows.synth(n, n, offs, seed=71)
    runs = case in ("stencil27", "runs2", *RUN_CASES)
    boffs = offs if runs else offs[::-1].copy()
    B = dg.DiaRows.synth(n, n, boffs, seed=72)
    plan = dg.SpmspmPlan(A, B)
    if case in ("stencil7", "band", "scatter"):   # shared-memory-tiled kernel
        assert plan.tile_rows > 0 and plan.tiled[1] > plan.tiled[0]
    if runs:     # register-blocked run-pair kernel
        assert plan.tile_rows < 0 and plan.tiled[1] > plan.tiled[0]
    Ct = plan.execute(A, B, plan.new_C())
    Cg = plan.execute(A, B, plan.new_C(), use_tiles=False)
    Cu = dg.spmspm(A, B, method="generic")
    assert np.array_equal(plan.C_off, Cu.offsets)
    ht, hg, hu = (x.vals.cpu().numpy() for x in (Ct, Cg, Cu))
    assert same(ht, hu) and same(hg, hu)
    # sub-ranges of rows, as the partitioned path calls them
    Cs = plan.new_C()
    for lo, hi in ((0, 1000), (1000, n // 2 + 7), (n // 2 + 7, n)):
        plan.execute(A, B, Cs, lo, hi)
    assert same(Cs.vals.cpu().numpy(), hu)


@pytest.mark.parametrize("case", list(RUN_CASES))
def test_runpair_b_window_shifts(case):
    """Row-window products whose B block starts at every residue mod 8 (as
    a partitioned product's halo does) match the whole product's rows bit
    for bit, with the run-pair kernel doing the interior."""
    n, offs = RUN_CASES[case]
    A = dg.DiaRows.synth(n, n, offs, seed=81)
    Cm = dg.spmspm(A, A)
    H = int(np.abs(offs).max())
    Ah = A.vals.cpu().numpy()
    for delta in range(8):
        lo, hi = n // 3 + delta, n // 3 + delta + 20_000
        wlo, whi = lo - H - delta, hi + H + 3
        Aw = dg.DiaRows.from_host(n, n, offs, Ah[:, wlo:whi], vrow0=wlo)
        Aa = dg.DiaRows.from_host(n, n, offs, Ah[:, lo:hi], vrow0=lo)
        plan = dg.SpmspmPlan(Aa, Aw)
        assert plan.tile_rows < 0 and plan.tiled[1] > plan.tiled[0], delta
        Cw = dg.DiaRows.empty(n, n, Cm.offsets, vrow0=lo, nrows=hi - lo)
        dg.spmspm(Aa, Aw, Cw)
        assert same(Cm.vals[:, lo:hi].cpu().numpy(), Cw.vals[:, :hi - lo].cpu().numpy()), delta


def test_runpair_misaligned_buffers_fall_back():
    """A C buffer that is not 32-byte aligned cannot take the run-pair
    kernel's vector stores; the plan must then run the generic kernel and
    still give the same values."""
    import ctypes
    n = 64 * 64 * 64
    offs = np.array([i + 64 * j + 4096 * k for k in (-1, 0, 1) for j in (-1, 0, 1)
                     for i in (-1, 0, 1)], np.int32)
    A = dg.DiaRows.synth(n, n, offs, seed=91)
    plan = dg.SpmspmPlan(A, A)
    assert plan.tile_rows < 0
    ref = plan.execute(A, A, plan.new_C())
    Cr = ref.vals
    flat = torch.zeros(Cr.numel() + 8, dtype=torch.float32, device="cuda")
    rc = dg.lib().dia_spmspm_plan_execute(plan._h, ctypes.c_void_p(A.vals.data_ptr()),
                                          ctypes.c_void_p(A.vals.data_ptr()),
                                          ctypes.c_void_p(flat.data_ptr() + 4), 0, n, 1,
                                          dg._stream())
    assert rc == 0
    torch.cuda.synchronize()
    got = flat[1:1 + Cr.numel()].view_as(Cr)
    assert same(Cr[:, :n].cpu().numpy(), got[:, :n].cpu().numpy())
