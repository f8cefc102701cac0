"""Complex64 DIA (dia_spmv_rows_c64, dia_expm_taylor_c64) against the CPU
oracle's restatement, bit for bit.  Pinned to the real, reference-pinned
path: with zero imaginary parts the complex SpMV equals the real SpMV (and
so the reference's CPU loop) bit for bit."""
import numpy as np
import pytest
import torch

import diagpu_b200 as dg
import oracle
from tests._util import same

pytestmark = pytest.mark.gpu


def _hermitian_band(n, offs, seed):
    """Rows-layout values of a Hermitian band: A[i, i+d] = conj(A[i+d, i])."""
    rng = np.random.default_rng(seed)
    offs = np.asarray(offs, np.int32)
    vals = np.zeros((len(offs), n), np.complex64)
    idx = {int(d): k for k, d in enumerate(offs)}
    for k, d in enumerate(offs):
        if d < 0:
            continue
        lo, hi = 0, n - d
        z = rng.uniform(-1, 1, hi - lo) + 1j * (rng.uniform(-1, 1, hi - lo) if d else 0)
        vals[k, lo:hi] = z
        if d:
            vals[idx[-d], d:d + hi - lo] = np.conj(z)
    return vals


def test_zero_imaginary_equals_real_spmv():
    n = 100_003
    offs = np.array([-1024, -7, -1, 0, 1, 7, 1024], np.int32)
    A = dg.DiaRows.synth(n, n, offs, seed=5)
    x = dg.synth_vector(n, seed=6)
    y_real = dg.spmv(A, x)[:n]
    Ac = dg.DiaRows.empty(n, n, offs, dtype=torch.complex64)
    Ac.vals.real.copy_(A.vals)
    yc = dg.spmv_c64(Ac, x.to(torch.complex64))
    assert same(yc.real.cpu().numpy(), y_real.cpu().numpy())
    assert (yc.imag == 0).all()


@pytest.mark.parametrize("n,offs", [(4096, [-64, -1, 0, 1, 64]), (1000, [-999, -3, 0, 5, 998]),
                                    (777, [0])])
def test_spmv_c64_equals_oracle(n, offs):
    rng = np.random.default_rng(n)
    offs = np.array(offs, np.int32)
    vals = (rng.standard_normal((len(offs), n)) + 1j * rng.standard_normal((len(offs), n)))
    for k, d in enumerate(offs):          # zero outside each diagonal, as the layout requires
        vals[k, :max(0, -d)] = 0
        vals[k, min(n, n - d):] = 0
    A = dg.DiaRows.from_host(n, n, offs, vals)
    x = (rng.standard_normal(n) + 1j * rng.standard_normal(n)).astype(np.complex64)
    y = dg.spmv_c64(A, torch.from_numpy(x).cuda()).cpu().numpy()
    ref = oracle.spmv_c64(offs, A.vals.cpu().numpy(), A.stride, x, n_rows=n, n_cols=n)
    assert same(y.view(np.float32), ref.view(np.float32))


@pytest.mark.parametrize("grid,t,m", [(64, 0.1, 16), (31, 0.5, 24)])
def test_schroedinger_evolution_equals_oracle(grid, t, m):
    n = grid * grid
    offs = np.array([-grid, -1, 0, 1, grid], np.int32)
    vals = _hermitian_band(n, offs, seed=grid)
    A = dg.DiaRows.from_host(n, n, offs, vals)
    rng = np.random.default_rng(3)
    x = (rng.standard_normal(n) + 1j * rng.standard_normal(n)).astype(np.complex64)
    y = dg.expm_taylor_c64(A, t, m, torch.from_numpy(x).cuda()).cpu().numpy()
    ref = oracle.expm_taylor_c64(offs, A.vals.cpu().numpy(), A.stride, t, m, x)
    assert same(y.view(np.float32), ref.view(np.float32))
    # a Hermitian generator evolves unitarily: the norm is kept to fp32 accuracy
    assert abs(np.linalg.norm(y) / np.linalg.norm(x) - 1) < 1e-5


def test_complex_entry_points_reject_real_values():
    A = dg.DiaRows.synth(64, 64, np.array([0], np.int32), seed=1)
    with pytest.raises(dg.DiaError):
        dg.spmv_c64(A, torch.zeros(64, dtype=torch.complex64, device="cuda"))


@pytest.mark.parametrize("n_rows,n_cols", [(1000, 1700), (2048, 513)])
def test_spmv_c64_rectangular(n_rows, n_cols):
    rng = np.random.default_rng(n_rows + n_cols)
    offs = np.array([-700, -2, 0, 3, 900], np.int32)
    vals = rng.standard_normal((len(offs), n_rows)) + 1j * rng.standard_normal((len(offs), n_rows))
    for k, d in enumerate(offs):
        rows = np.arange(n_rows)
        vals[k, (rows + d < 0) | (rows + d >= n_cols)] = 0
    A = dg.DiaRows.from_host(n_rows, n_cols, offs, vals)
    x = (rng.standard_normal(n_cols) + 1j * rng.standard_normal(n_cols)).astype(np.complex64)
    y = dg.spmv_c64(A, torch.from_numpy(x).cuda()).cpu().numpy()
    ref = oracle.spmv_c64(offs, A.vals.cpu().numpy(), A.stride, x, n_rows=n_rows, n_cols=n_cols)
    assert same(y.view(np.float32), ref.view(np.float32))
