"""Device-side symbolic phase and matrix-power chains (dia_spmspm_symbolic_device,
dia_spmspm_rows_device, diagpu_b200.PowerChain).

The output offset set must equal the host symbolic phase (itself pinned to
the reference's make_c_structure) bit for bit, and every power of a chain
must equal the host-planned product of the previous power with H, and the
CPU oracle, bit for bit (same pair order, separately rounded multiply and
add)."""
import numpy as np
import pytest
import torch

import diagpu_b200 as dg
import oracle
from tests._util import dev, rows_to_hm, same

pytestmark = pytest.mark.gpu


def _device_sumset(n, A_off, B_off, cap, a_cap=None):
    A_off = np.asarray(A_off, np.int32)
    a_cap = len(A_off) if a_cap is None else a_cap
    dA = torch.zeros(max(a_cap, 1), dtype=torch.int32, device="cuda")
    dA[:len(A_off)] = dev(A_off)
    nA = dev(np.array([len(A_off)], np.int32))
    C_off, nC = dg.spmspm_symbolic_device(n, dA, nA, a_cap, dev(np.asarray(B_off, np.int32)), cap)
    torch.cuda.synchronize()
    return C_off.cpu().numpy(), int(nC.item())


@pytest.mark.parametrize("case", ["stencil", "scatter", "edges", "tiny", "single", "large_n"])
def test_symbolic_device_equals_host(case):
    rng = np.random.default_rng(5)
    if case == "stencil":
        n, A, B = 4096, [-64, -1, 0, 1, 64], [-64, -1, 0, 1, 64]
    elif case == "scatter":
        n = 100_000
        A = np.unique(rng.integers(-900, 901, 40))
        B = np.unique(rng.integers(-700, 701, 30))
    elif case == "edges":       # sums that leave (-n, n) are dropped
        n, A, B = 1000, [-999, -500, 0, 998, 999], [-999, -1, 0, 1, 999]
    elif case == "tiny":
        n, A, B = 3, [-2, 0, 1], [-1, 2]
    elif case == "single":
        n, A, B = 17, [0], [5]
    else:                       # bitmap over 2n-1 = 268M offsets, several scan blocks
        n = 1 << 27
        A = [-65793, -256, 0, 256, 65793]
        B = [-(1 << 26), -3, 0, 7, (1 << 26) + 5]
    A, B = np.asarray(A, np.int32), np.asarray(B, np.int32)
    ref = dg.spmspm_symbolic(n, A, B)["C_off"]
    got, nc = _device_sumset(n, A, B, cap=len(A) * len(B) + 3)
    assert nc == len(ref)
    assert np.array_equal(got[:nc], ref)


def test_symbolic_device_capacity_overflow_is_reported():
    n, A, B = 4096, np.arange(-20, 21, dtype=np.int32), np.arange(-10, 11, dtype=np.int32)
    ref = dg.spmspm_symbolic(n, A, B)["C_off"]
    got, nc = _device_sumset(n, A, B, cap=16)
    assert nc == len(ref) > 16            # the true count, above the capacity
    assert np.array_equal(got[:16], ref[:16])


def test_symbolic_device_reads_count_from_device():
    """Entries of A's offset buffer past the device count are ignored."""
    n = 5000
    A = np.array([-7, 0, 3, 4000, -4000], np.int32)
    dA = dev(A)
    nA = dev(np.array([3], np.int32))      # only the first three are live
    B = np.array([-2, 0, 2], np.int32)
    C_off, nC = dg.spmspm_symbolic_device(n, dA, nA, len(A), dev(B), 64)
    ref = dg.spmspm_symbolic(n, A[:3], B)["C_off"]
    assert int(nC.item()) == len(ref)
    assert np.array_equal(C_off.cpu().numpy()[:len(ref)], ref)


def _oracle_product(n, A, B):
    a = rows_to_hm(n, A.offsets, A.vals.cpu().numpy())
    b = rows_to_hm(n, B.offsets, B.vals.cpu().numpy())
    off, ln, st = oracle.c_structure(n, A.offsets, B.offsets)
    return off, oracle.dia_spgemm_hm(n, (A.offsets, *a), (B.offsets, *b), (off, ln, st))


@pytest.mark.parametrize("grid,k", [(64, 5), (37, 4)])
def test_power_chain_equals_host_products_and_oracle(grid, k):
    """H = 2D 5-point stencil (odd grid: ragged diagonals); P_k = H^k."""
    n = grid * grid
    H = dg.DiaRows.synth(n, n, np.array([-grid, -1, 0, 1, grid], np.int32), seed=31)
    chain = dg.PowerChain(H, max_diags=4 * k * k + 8)
    P = H
    for step in range(2, k + 1):
        chain.step()
        got = chain.power()
        P_prev, P = P, dg.spmspm(P, H)    # host-planned product of the previous power
        assert np.array_equal(got.offsets, P.offsets), step
        assert same(got.vals[:, :n].cpu().numpy(), P.vals[:, :n].cpu().numpy()), step
        # padding outside each diagonal is exactly zero
        for j, d in enumerate(got.offsets):
            row = got.vals[j].cpu().numpy()
            lo, hi = max(0, -int(d)), min(n, n - int(d))
            assert (row[:lo] == 0).all() and (row[hi:n] == 0).all()
    # the last power against the CPU oracle applied to the previous one
    off, ref = _oracle_product(n, P_prev, H)
    assert np.array_equal(off, got.offsets)
    assert same(rows_to_hm(n, got.offsets, got.vals.cpu().numpy())[2], ref)


def test_power_chain_capacity_error():
    n = 1024
    H = dg.DiaRows.synth(n, n, np.array([-32, -1, 0, 1, 32], np.int32), seed=3)
    chain = dg.PowerChain(H, max_diags=10)
    chain.step()                          # H^2 has 13 diagonals
    with pytest.raises(dg.DiaError) as e:
        chain.power()
    assert e.value.code == dg.DIA_ERR_CAPACITY


def test_power_chain_has_no_host_sync():
    """Steps only enqueue work: all k steps are queued while the first is
    still waiting behind a long kernel on the stream."""
    n = 1 << 16
    H = dg.DiaRows.synth(n, n, np.array([-256, -1, 0, 1, 256], np.int32), seed=9)
    chain = dg.PowerChain(H, max_diags=64)
    torch.cuda.synchronize()
    torch.cuda._sleep(200_000_000)        # ~0.1 s of GPU time ahead of the steps
    ev = torch.cuda.Event()
    for _ in range(4):
        chain.step()
    ev.record()
    assert not ev.query()                 # nothing forced the host to wait
    torch.cuda.synchronize()
    assert chain.power().K == 61          # H^5: offsets 256a + b with |a| + |b| <= 5


def test_symbolic_device_fuzz():
    """Random sizes and offset sets, sums that fall outside (-n, n) included."""
    rng = np.random.default_rng(2024)
    for _ in range(40):
        n = int(rng.integers(1, 3000))
        na, nb = int(rng.integers(1, 40)), int(rng.integers(1, 12))
        A = np.unique(rng.integers(-(n - 1), n, na)).astype(np.int32)
        B = np.unique(rng.integers(-(n - 1), n, nb)).astype(np.int32)
        ref = dg.spmspm_symbolic(n, A, B)["C_off"]
        got, nc = _device_sumset(n, A, B, cap=len(A) * len(B) + 1, a_cap=len(A) + 5)
        assert nc == len(ref) and np.array_equal(got[:nc], ref), (n, A, B)


def test_power_chain_offsets_reach_the_matrix_edge():
    """Powers whose sums leave (-n, n): those diagonals are dropped exactly as
    the host symbolic phase drops them, values still equal the host path."""
    n = 300
    H = dg.DiaRows.synth(n, n, np.array([-120, -1, 0, 2, 150], np.int32), seed=8)
    chain = dg.PowerChain(H, max_diags=200)
    P = H
    for _ in range(3):
        chain.step()
        P = dg.spmspm(P, H)
        got = chain.power()
        assert np.abs(got.offsets).max() < n
        assert np.array_equal(got.offsets, P.offsets)
        assert same(got.vals[:, :n].cpu().numpy(), P.vals[:, :n].cpu().numpy())
