"""Lanczos on the device (dia_lanczos): the tridiagonal and the Lanczos
vectors equal the CPU oracle's recurrence (fp32 vectors bit for bit, fp64
coefficients to 1e-12 relative: the same exact products summed in another
order), and the Ritz values converge to the operator's extreme eigenvalues."""
import numpy as np
import pytest
import torch

import diagpu_b200 as dg
import oracle
from tests._util import same
from tests.test_oracle import _sym_band

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("g,m", [(20, 60), (64, 40), (37, 25)])
def test_lanczos_equals_oracle(g, m):
    offs, vals, stride, A = _sym_band(g, g)
    n = g * g
    D = dg.DiaRows.from_host(n, n, offs, vals[:, :n])
    x = np.random.default_rng(g).uniform(-1, 1, n).astype(np.float32)
    al, be, B = dg.lanczos(D, m, torch.from_numpy(x).cuda(), basis=True)
    ral, rbe, rB = oracle.lanczos(offs, D.vals.cpu().numpy(), D.stride, m, x, basis=True)
    assert np.allclose(al.cpu().numpy(), ral, rtol=1e-12, atol=1e-12)
    assert np.allclose(be.cpu().numpy(), rbe, rtol=1e-12, atol=1e-12)
    assert same(B.cpu().numpy(), rB)
    if g == 20:
        al = al.cpu().numpy()
        be = be.cpu().numpy()
        T = np.diag(al) + np.diag(be[:-1], 1) + np.diag(be[:-1], -1)
        ev, ea = np.linalg.eigvalsh(T), np.linalg.eigvalsh(A)
        assert abs(ev.max() - ea.max()) / abs(ea.max()) < 1e-5


def test_lanczos_config1_operator_runs_without_sync():
    """Config-1 operator (n = 2^20, symmetric): 30 steps queue behind a long
    kernel without the host waiting; the largest Ritz value approaches the
    bound 8 of the 5-point operator."""
    n = 1 << 20
    offs = np.array([-1024, -1, 0, 1, 1024], np.int32)
    D = dg.DiaRows.empty(n, n, offs)
    for k, (d, b) in enumerate(zip(offs, (-1.0, -1.0, 4.0, -1.0, -1.0))):
        lo, hi = max(0, -int(d)), min(n, n - int(d))
        D.vals[k, lo:hi] = b
    x = dg.synth_vector(n, seed=5)
    torch.cuda.synchronize()
    torch.cuda._sleep(200_000_000)
    al, be = dg.lanczos(D, 30, x)
    ev = torch.cuda.Event()
    ev.record()
    assert not ev.query()
    torch.cuda.synchronize()
    a, b = al.cpu().numpy(), be.cpu().numpy()
    T = np.diag(a) + np.diag(b[:-1], 1) + np.diag(b[:-1], -1)
    assert 7.5 < np.linalg.eigvalsh(T).max() <= 8.0 + 1e-6
