"""SpMV parity on the GPU (through the C ABI) against the oracle and the
reference's golden outputs.  FP32, same summation order: results must be
equal, not merely close (relative L2 <= 1e-6, is
checked as well)."""
import ctypes as C

import numpy as np
import pytest
import torch

import diagpu_b200 as dg
import oracle
from tests._util import dev, rel_l2, same

pytestmark = pytest.mark.gpu


def test_kat5_recon(golden):
    g = golden["spmv_kat5"]
    y = dg.spmv_recon(5, 5, dev(g["recon_off"]), dev(g["recon"]), dev(g["x"]))
    assert same(y.cpu().numpy(), g["y"])


def test_reference_cases_recon(golden):
    g = golden["spmv_cases"]
    for name in g["names"]:
        rec = g[f"{name}__recon"]
        N = rec.shape[1]
        y = dg.spmv_recon(N, N, dev(g[f"{name}__recon_off"]), dev(rec), dev(g[f"{name}__x"]))
        assert same(y.cpu().numpy(), g[f"{name}__y"]), name


class ReconView(C.Structure):
    _fields_ = [("rows", C.c_int), ("cols", C.c_int), ("num_diags", C.c_int),
                ("diag_offsets", C.c_void_p), ("values", C.c_void_p)]


def test_cxx_dropin_launcher(golden):
    """launch_tc_spmv_regdirect with the reference's exact signature."""
    g = golden["spmv_cases"]
    fn = getattr(dg.lib(), "_Z24launch_tc_spmv_regdirect9ReconViewPKfiPfP11CUstream_st")
    fn.argtypes = [ReconView, C.c_void_p, C.c_int, C.c_void_p, C.c_void_p]
    fn.restype = None
    name = "wide9"
    rec, off, x = g[f"{name}__recon"], dev(g[f"{name}__recon_off"]), dev(g[f"{name}__x"])
    drec = dev(rec)
    N = rec.shape[1]
    y = torch.full((N,), 7.0, device="cuda")
    fn(ReconView(N, N, len(off), off.data_ptr(), drec.data_ptr()), x.data_ptr(), N, y.data_ptr(),
       torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert same(y.cpu().numpy(), g[f"{name}__y"])


def test_recon_xsize_and_rectangular():
    rng = np.random.default_rng(1)
    rows, cols, K = 300, 257, 6
    offs = np.array([200, 9, 0, -3, -40, -299], np.int32)
    rec = rng.standard_normal((K, cols)).astype(np.float32)
    x = rng.standard_normal(cols).astype(np.float32)
    for xs in (cols, 100):
        y = dg.spmv_recon(rows, cols, dev(offs), dev(rec), dev(x), x_size=xs)
        ref = oracle.spmv_recon(rows, cols, offs, rec, x, x_size=xs)
        assert same(y.cpu().numpy(), ref)


@pytest.mark.parametrize("n,offs", [
    (1, [0]), (37, [-1, 0, 1]), (1000, [-999, -500, 0, 3, 999]), (5000, []),
    (70000, list(range(-200, 201))),            # > one shared-memory term chunk
    (4099, [-4100, -33, 5, 4200]),               # offsets beyond the matrix
])
def test_rows_layout_vs_oracle(n, offs):
    A = dg.DiaRows.synth(n, n, np.array(offs, np.int32), seed=11)
    x = dg.synth_vector(n, seed=12)
    y = dg.spmv(A, x)[:n]
    ref = oracle.spmv_rowidx(np.array(offs, np.int32), A.vals.cpu().numpy(), A.stride,
                             x.cpu().numpy(), ncols=n, nrows=n)
    assert same(y.cpu().numpy(), ref)


def test_rows_subranges_and_x_window():
    n, offs = 50000, np.array([-7000, -1, 0, 1, 6500], np.int32)
    A = dg.DiaRows.synth(n, n, offs, seed=3)
    x = dg.synth_vector(n, seed=4)
    full = dg.spmv(A, x).cpu().numpy()[:n]
    # rows [20000, 30000) with x restricted to the window they touch
    lo, hi = 20000, 30000
    xw = x[lo - 7000:hi + 6500].contiguous()
    y = torch.full((A.stride,), -5.0, device="cuda")
    dg.spmv(A, xw, y, x_lo=lo - 7000, row_lo=lo, row_hi=hi)
    yh = y.cpu().numpy()
    assert same(yh[lo:hi], full[lo:hi])
    assert (yh[:lo] == -5.0).all() and (yh[hi:] == -5.0).all()


def test_synth_matches_oracle_bitwise():
    offs = np.array([-70000, -3, 0, 11, 65537], np.int32)
    A = dg.DiaRows.synth(300000, 300000, offs, seed=99, base=[0, -1, 4, -1, 0], lo=-0.01,
                         hi=0.01, vrow0=100000, nrows=123456)
    ref = oracle.synth_rowidx(99, 300000, 300000, offs, base=np.array([0, -1, 4, -1, 0],
                              np.float32), lo=-0.01, hi=0.01, row0=100000, nrows=123456)
    assert np.array_equal(A.vals.cpu().numpy(), ref)
    B = dg.DiaRows.synth(5000, 5000, offs[1:4], seed=5, kind=1, lo=0.0, hi=1.0)
    refB = oracle.synth_rowidx(5, 5000, 5000, offs[1:4], kind=1, lo=0.0, hi=1.0)
    assert np.array_equal(B.vals.cpu().numpy(), refB)
    assert np.array_equal(dg.synth_vector(1000, 8, i0=77).cpu().numpy(),
                          oracle.synth_vector(8, 1000, i0=77))


def test_config1_poisson_full():
    """Config 1: 2D 5-point Poisson, n = 1024^2, full-size parity."""
    n = 1 << 20
    offs = np.array([-1024, -1, 0, 1, 1024], np.int32)
    base = np.array([-1, -1, 4, -1, -1], np.float32)
    A = dg.DiaRows.synth(n, n, offs, seed=101, base=base, lo=-0.01, hi=0.01)
    x = dg.synth_vector(n, seed=102)
    y = dg.spmv(A, x)[:n].cpu().numpy()
    ref = oracle.spmv_rowidx(offs, A.vals.cpu().numpy(), A.stride, x.cpu().numpy(), ncols=n,
                             nrows=n)
    assert same(y, ref)
    assert rel_l2(y, ref) <= 1e-6


def test_config5_windows():
    """Config 5 (n = 67M, 27 diagonals) at full size, checked on windows at
    both ends, the middle and the +-65536 clusters against the oracle run
    on the same generated rows."""
    n = 256 * 256 * 1024
    offs = np.array([i + 256 * j + 65536 * k for k in (-1, 0, 1) for j in (-1, 0, 1)
                     for i in (-1, 0, 1)], np.int32)
    A = dg.DiaRows.synth(n, n, offs, seed=501)
    x = dg.synth_vector(n, seed=502)
    y = dg.spmv(A, x)
    for lo in (0, 65000, n // 2 + 13, n - 70000, n - 4096):
        hi = min(n, lo + 4096)
        rows = oracle.synth_rowidx(501, n, n, offs, row0=lo, nrows=hi - lo)
        xlo, xhi = max(0, lo - 65793), min(n, hi + 65793)
        xw = oracle.synth_vector(502, xhi - xlo, i0=xlo)
        ref = oracle.spmv_rowidx(offs, rows, rows.shape[1], xw, ncols=n, row0=lo, nrows=hi - lo,
                                 x_lo=xlo)
        assert same(y[lo:hi].cpu().numpy(), ref), lo
