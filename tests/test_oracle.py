"""The CPU oracle restatement against the reference's own outputs (golden
fixtures made by tests/golden/make_golden.py from the compiled reference)."""
import numpy as np
import pytest

import oracle


def _case(npz, name, key):
    return npz[f"{name}__{key}"]


def test_kat5_recon_and_spmv(golden):
    g = golden["spmv_kat5"]
    off, rec = oracle.build_recon(5, 5, g["dia_off"], g["dia_start"], g["dia_len"], g["dia_val"])
    assert (off == g["recon_off"]).all()
    assert np.array_equal(rec, g["recon"])
    y = oracle.spmv_recon(5, 5, off, rec, g["x"])
    assert np.array_equal(y, g["y"])
    assert np.array_equal(y, g["y_dense"])  # small integers: exact


def test_spmv_cases(golden):
    g = golden["spmv_cases"]
    for name in g["names"]:
        H, x = _case(g, name, "H"), _case(g, name, "x")
        N = H.shape[0]
        off, rec = _case(g, name, "recon_off"), _case(g, name, "recon")
        y = oracle.spmv_recon(N, N, off, rec, x)
        assert np.array_equal(y, _case(g, name, "y")), name
        # same sum on the rows layout with the recon (descending) order
        rows = np.zeros((len(off), N), np.float32)
        for k, d in enumerate(off):
            for i in range(N):
                if 0 <= i + d < N:
                    rows[k, i] = H[i, i + d]
        y2 = oracle.spmv_rowidx(off, rows, N, x, ncols=N)
        assert np.array_equal(y2, _case(g, name, "y")), name


def _hm(g, name, tag):
    return tuple(g[f"{name}__{tag}_{f}"] for f in ("off", "len", "start", "val"))


@pytest.mark.parametrize("fixture", ["spmspm_banded", "spmspm_scatter"])
def test_spmspm_structure_and_values(golden, fixture):
    g = golden[fixture]
    for name in g["names"]:
        A, B = _hm(g, name, "A"), _hm(g, name, "B")
        n = int(A[1].max()) if len(A[1]) else 0
        n = int(max(A[1][A[0] == 0])) if (A[0] == 0).any() else n
        off, ln, st = oracle.c_structure(n, A[0], B[0])
        assert (off == g[f"{name}__C_off"]).all(), name
        assert (ln == g[f"{name}__C_len"]).all(), name
        assert (st == g[f"{name}__C_start"]).all(), name
        C = oracle.dia_spgemm_hm(n, A, B, (off, ln, st))
        assert np.array_equal(C, g[f"{name}__C_val"]), name
        if f"{name}__C_dense" in g:
            ref = g[f"{name}__C_dense"]
            assert np.abs(C - ref).max() <= 1e-5 * max(1.0, np.abs(ref).max()), name


def test_gemm_diag_layout_and_values(golden):
    g = golden["gemm_diag"]
    for name in g["names"]:
        off = g[f"{name}__off"]
        n = g[f"{name}__DA"].size // len(off)
        co, cl, k2i, kl, tot = oracle.build_c_layout(n, off, off)
        assert (co == g[f"{name}__C_offsets"]).all()
        assert (cl == g[f"{name}__C_lens"]).all()
        assert (k2i == g[f"{name}__k_to_idx"]).all()
        assert (kl == g[f"{name}__k_list"]).all()
        C32, _ = oracle.gemm_diag(g[f"{name}__DA"], off, g[f"{name}__DB"], off, n, f64=False)
        assert np.array_equal(C32, g[f"{name}__C"]), name
        C64, _ = oracle.gemm_diag(g[f"{name}__DA"], off, g[f"{name}__DB"], off, n, f64=True)
        rel = np.linalg.norm(C64 - g[f"{name}__C"]) / np.linalg.norm(C64)
        assert rel < 1e-6, name


def test_pair_lists_order():
    ptr, pa, pb = oracle.pair_lists(100, [-1, 0, 1], [1, 0, -1], [-2, -1, 0, 1, 2])
    assert list(ptr) == [0, 1, 3, 6, 8, 9]
    assert list(pa) == [0, 0, 1, 0, 1, 2, 1, 2, 2]


def test_synth_deterministic_and_partition_free():
    offs = [-3, 0, 5]
    full = oracle.synth_rowidx(7, 100, 100, offs)
    part = oracle.synth_rowidx(7, 100, 100, offs, row0=40, nrows=30)
    assert np.array_equal(full[:, 40:70], part[:, :30])
    assert (full[0, :3] == 0).all() and (full[2, 95:100] == 0).all()
    assert np.abs(full).max() <= 1.0
    nrm = oracle.synth_rowidx(9, 20000, 20000, [0], kind=1, lo=0.0, hi=1.0)[0, :20000]
    assert abs(nrm.mean()) < 0.05 and abs(nrm.std() - 1.0) < 0.05


def test_expm_taylor_oracle_matches_matrix_exponential():
    """The Taylor recurrence the library follows converges to exp(tA) x
    (scipy's expm on the dense matrix), so the definition is pinned."""
    import scipy.linalg as sl
    rng = np.random.default_rng(0)
    n, stride = 96, 96
    offs = np.array([-8, -1, 0, 1, 8], np.int32)
    vals = np.zeros((len(offs), stride), np.float32)
    A = np.zeros((n, n))
    for k, d in enumerate(offs):
        lo, hi = max(0, -d), min(n, n - d)
        vals[k, lo:hi] = rng.uniform(-1, 1, hi - lo)
        A[np.arange(lo, hi), np.arange(lo, hi) + d] = vals[k, lo:hi]
    x = rng.uniform(-1, 1, n).astype(np.float32)
    for t, m in ((0.1, 12), (0.5, 20)):
        y = oracle.expm_taylor(offs, vals, stride, t, m, x)
        ref = sl.expm(t * A) @ x
        assert np.linalg.norm(y - ref) / np.linalg.norm(ref) < 1e-6
    # m = 0 is the identity
    assert np.array_equal(oracle.expm_taylor(offs, vals, stride, 0.3, 0, x), x)


def test_expm_taylor_c64_oracle_matches_matrix_exponential():
    """exp(-i t H) x of a Hermitian band: the recurrence converges to scipy's
    expm and keeps the norm (unitary evolution)."""
    import scipy.linalg as sl
    rng = np.random.default_rng(1)
    n, stride = 80, 96
    offs = np.array([-7, -1, 0, 1, 7], np.int32)
    H = np.zeros((n, n), np.complex128)
    for d in (0, 1, 7):
        for i in range(n - d):
            z = complex(rng.uniform(-1, 1), rng.uniform(-1, 1) if d else 0.0)
            H[i, i + d] = z
            H[i + d, i] = np.conj(z)
    vals = np.zeros((len(offs), stride), np.complex64)
    for k, d in enumerate(offs):
        for i in range(max(0, -d), min(n, n - d)):
            vals[k, i] = H[i, i + d]
    x = (rng.uniform(-1, 1, n) + 1j * rng.uniform(-1, 1, n)).astype(np.complex64)
    y = oracle.expm_taylor_c64(offs, vals, stride, 0.3, 20, x)
    ref = sl.expm(-1j * 0.3 * H) @ x
    assert np.linalg.norm(y - ref) / np.linalg.norm(ref) < 1e-6
    assert abs(np.linalg.norm(y) / np.linalg.norm(x) - 1) < 1e-6
    yv = oracle.spmv_c64(offs, vals, stride, x, n_rows=n, n_cols=n)
    assert np.linalg.norm(yv - H @ x) / np.linalg.norm(H @ x) < 1e-6


def _sym_band(g, seed):
    """Rows-layout values of a symmetric 2D 5-point-type band on a g x g grid."""
    n, stride = g * g, (g * g + 31) // 32 * 32
    offs = np.array([-g, -1, 0, 1, g], np.int32)
    rng = np.random.default_rng(seed)
    vals = np.zeros((5, stride), np.float32)
    for k, (d, b) in enumerate(zip(offs, (-1, -1, 4, -1, -1))):
        lo, hi = max(0, -d), min(n, n - d)
        vals[k, lo:hi] = b + rng.uniform(-0.01, 0.01, hi - lo)
    for k, d in enumerate(offs):           # A[i, i+d] = A[i+d, i]
        if d > 0:
            vals[list(offs).index(-d), d:n] = vals[k, 0:n - d]
    A = np.zeros((n, n))
    for k, d in enumerate(offs):
        i = np.arange(max(0, -d), min(n, n - d))
        A[i, i + d] = vals[k, i]
    return offs, vals, stride, A


def test_lanczos_oracle_finds_extreme_eigenvalues():
    """The Lanczos recurrence the library follows: its tridiagonal's extreme
    eigenvalues converge to the operator's (numpy eigvalsh on the dense
    matrix)."""
    offs, vals, stride, A = _sym_band(20, 0)
    assert np.array_equal(A, A.T)
    x = np.random.default_rng(1).uniform(-1, 1, A.shape[0]).astype(np.float32)
    al, be = oracle.lanczos(offs, vals, stride, 60, x)
    T = np.diag(al) + np.diag(be[:-1], 1) + np.diag(be[:-1], -1)
    ev, ea = np.linalg.eigvalsh(T), np.linalg.eigvalsh(A)
    assert abs(ev.max() - ea.max()) / abs(ea.max()) < 1e-5
    assert abs(ev.min() - ea.min()) / abs(ea.max()) < 1e-5
