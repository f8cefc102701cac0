"""Truncated-Taylor time evolution y = sum_j (tA)^j x / j! (dia_expm_taylor):
the chained SpMV driver equals the CPU oracle's recurrence bit for bit."""
import numpy as np
import pytest
import torch

import diagpu_b200 as dg
import oracle
from tests._util import same

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("grid,t,m", [(64, 0.05, 12), (37, 0.2, 20), (8, 1.0, 1), (8, 0.3, 0)])
def test_expm_taylor_equals_oracle(grid, t, m):
    n = grid * grid
    offs = np.array([-grid, -1, 0, 1, grid], np.int32)
    A = dg.DiaRows.synth(n, n, offs, seed=41, base=[-1, -1, 4, -1, -1], lo=-0.01, hi=0.01)
    x = dg.synth_vector(n, seed=42)
    y = dg.expm_taylor(A, t, m, x)
    ref = oracle.expm_taylor(offs, A.vals.cpu().numpy(), A.stride, t, m, x.cpu().numpy())
    assert same(y.cpu().numpy(), ref)


def test_expm_taylor_config1_size_and_graph_capture():
    """Config-1 operator (n = 2^20): a captured CUDA graph of the driver
    replays to the same bits as the eager call and the oracle."""
    n = 1 << 20
    offs = np.array([-1024, -1, 0, 1, 1024], np.int32)
    A = dg.DiaRows.synth(n, n, offs, seed=101, base=[-1, -1, 4, -1, -1], lo=-0.01, hi=0.01)
    x = dg.synth_vector(n, seed=102)
    y0 = dg.expm_taylor(A, 0.01, 16, x)
    ref = oracle.expm_taylor(offs, A.vals.cpu().numpy(), A.stride, 0.01, 16, x.cpu().numpy())
    assert same(y0.cpu().numpy(), ref)
    y = torch.empty(n, device="cuda")
    work = torch.empty(2 * n, device="cuda")
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        dg.expm_taylor(A, 0.01, 16, x, y, work=work)     # warm-up on the capture stream
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        dg.expm_taylor(A, 0.01, 16, x, y, work=work)
    y.zero_()
    g.replay()
    torch.cuda.synchronize()
    assert same(y.cpu().numpy(), ref)


def test_expm_taylor_rejects_partial_blocks():
    n = 256
    A = dg.DiaRows.synth(n, n, np.array([0], np.int32), seed=1, vrow0=64, nrows=64)
    with pytest.raises(dg.DiaError):
        dg.expm_taylor(A, 0.1, 3, torch.zeros(n, device="cuda"))


def test_expm_taylor_negative_time_many_terms():
    n = 3000
    offs = np.array([-50, -1, 0, 1, 50], np.int32)
    A = dg.DiaRows.synth(n, n, offs, seed=43)
    x = dg.synth_vector(n, seed=44)
    y = dg.expm_taylor(A, -0.2, 30, x)
    ref = oracle.expm_taylor(offs, A.vals.cpu().numpy(), A.stride, -0.2, 30, x.cpu().numpy())
    assert same(y.cpu().numpy(), ref)
