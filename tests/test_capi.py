"""Host-side checks of the C ABI (no GPU): the library loads, exports every
symbol include/*.h declares, validates arguments, and its symbolic phase
matches the oracle bit for bit."""
import ctypes as C
import os
import re

import numpy as np
import pytest

import diagpu_b200 as dg
import oracle

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    syms = set()
    for f in os.listdir(os.path.join(ROOT, "include")):
        src = open(os.path.join(ROOT, "include", f)).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        for m in re.finditer(r"\b(dia_\w+)\s*\(", src):
            syms.add(m.group(1))
    return syms


def test_exports_every_declared_symbol():
    L = dg.lib()
    syms = declared_symbols()
    assert "dia_spmv_recon" in syms and "dia_gemm_diag" in syms
    for s in syms:
        assert hasattr(L, s), s
    # C++ drop-in with the reference's mangled signature
    out = os.popen(f"nm -D {dg.LIB_PATH}").read()
    assert "_Z24launch_tc_spmv_regdirect9ReconViewPKfiPfP11CUstream_st" in out


def test_argument_validation_without_gpu():
    L = dg.lib()
    assert L.dia_spmv_recon(-1, 4, 1, None, None, None, 4, None, None) == dg.DIA_ERR_INVALID
    assert "negative" in L.dia_last_error().decode()
    assert L.dia_spmv_recon(0, 4, 1, None, None, None, 4, None, None) == dg.DIA_OK
    assert L.dia_gemm_diag_ex(None, None, None, None, None, None, 1, 1, 4, None, None, None,
                              None, 2, 0, None) == dg.DIA_ERR_INVALID


CASES = [
    (2097152, [0, 1, -1, 128, -128, 16384, -16384], None),
    (1000, list(range(-16, 17)), list(range(-16, 17))),
    (20, list(range(-16, 17)), [3, -7, 0]),
    (1, [0], [0]),
    (5, [4, -4], [4, -4]),
]


@pytest.mark.parametrize("n,A,B", CASES)
def test_symbolic_matches_oracle(n, A, B):
    B = A if B is None else B
    A = [a for a in A if abs(a) < n] or [0]
    r = dg.spmspm_symbolic(n, A, B)
    off, ln, st = oracle.c_structure(n, A, B)
    assert np.array_equal(r["C_off"], off)
    assert np.array_equal(r["C_len"], ln)
    assert np.array_equal(r["C_start"], st)
    ptr, pa, pb = oracle.pair_lists(n, A, B, off)
    assert np.array_equal(r["pair_ptr"], ptr)
    assert np.array_equal(r["pair_a"], pa) and np.array_equal(r["pair_b"], pb)


def test_symbolic_config5_structure():
    offs = [i + 256 * j + 65536 * k for k in (-1, 0, 1) for j in (-1, 0, 1) for i in (-1, 0, 1)]
    r = dg.spmspm_symbolic(67108864, offs, offs)
    assert len(r["C_off"]) == 125 and len(r["pair_a"]) == 729
    assert int(r["C_len"].astype(np.int64).sum()) == 8378769914


def test_symbolic_rejects_repeats_and_small_buffers():
    with pytest.raises(dg.DiaError):
        dg.spmspm_symbolic(10, [0, 0], [1])
    L = dg.lib()
    A = np.array([0, 1], np.int32)
    nc, npairs = C.c_int(1), C.c_int64(100)
    off = np.zeros(1, np.int32)
    rc = L.dia_spmspm_symbolic(10, A.ctypes.data_as(C.c_void_p), 2, A.ctypes.data_as(C.c_void_p),
                               2, C.byref(nc), off.ctypes.data_as(C.c_void_p), None, None,
                               C.byref(npairs), None, None, None)
    assert rc == dg.DIA_ERR_CAPACITY and nc.value == 3 and npairs.value == 4


def test_halo_plan_partition():
    from diagpu_b200 import dist
    parts = [dist.row_block(67108864, 8, r) for r in range(8)]
    assert parts[0][0] == 0 and parts[-1][1] == 67108864
    assert all(parts[i][1] == parts[i + 1][0] for i in range(7))
    assert all((p[1] - p[0]) % 32 == 0 for p in parts[:-1])


def test_validation_returns_status_not_exit():
    """Invalid calls return DIA_ERR_* with a message; nothing reaches the
    GPU (these run without one)."""
    L = dg.lib()
    p = C.c_void_p
    # rows outside the stored block
    rc = L.dia_spmv_rows(100, 100, 1, p(8), p(8), 32, 0, 0, 100, p(8), 0, 100, p(8), None)
    assert rc == dg.DIA_ERR_INVALID and "outside the stored block" in L.dia_last_error().decode()
    # rows x cols beyond int32
    rc = L.dia_spmv_rows(1 << 31, 10, 1, p(8), p(8), 1 << 32, 0, 0, 10, p(8), 0, 10, p(8), None)
    assert rc in (dg.DIA_ERR_UNSUPPORTED, dg.DIA_ERR_INVALID)
    # SpMSpM over the rows layout: B rows outside its buffer
    rc = L.dia_spmspm_rows(100, p(8), 128, p(8), 1, p(8), 128, 0, -5, 100, p(8), 1, p(8), 128,
                           p(8), 1, 0, 0, 100, None)
    assert rc == dg.DIA_ERR_INVALID
    # planned product: geometry outside the buffers is rejected before any allocation
    plan = C.c_void_p()
    one = np.array([0], np.int32)
    ptr = one.ctypes.data_as(C.c_void_p)
    rc = L.dia_spmspm_plan_create(100, ptr, 1, ptr, 1, 32, 128, 128, 0, 100, 0, 0, 100,
                                  C.byref(plan))
    assert rc == dg.DIA_ERR_INVALID and not plan.value
    # null handles
    assert L.dia_spmspm_plan_execute(None, None, None, None, 0, 1, 1, None) == dg.DIA_ERR_INVALID
    assert L.dia_dist_spmv_step(None, 1, 1, 1, None, None, 32, 0, None, 0, 1, None, None, 0, 1,
                                0, 1, 0, None) == dg.DIA_ERR_INVALID
    assert L.dia_dist_create(0, 0, None, C.byref(C.c_void_p())) == dg.DIA_ERR_INVALID
    assert L.dia_device_status(None, 0) == dg.DIA_ERR_INVALID


def test_symbolic_fuzz_against_oracle():
    """Random sizes and offset sets (storage order unsorted, sums leaving
    (-n, n)): structure and pair lists equal the reference restatement."""
    rng = np.random.default_rng(99)
    for _ in range(60):
        n = int(rng.integers(1, 5000))
        A = rng.permutation(np.unique(rng.integers(-(n - 1), n, int(rng.integers(1, 30)))))
        B = rng.permutation(np.unique(rng.integers(-(n - 1), n, int(rng.integers(1, 30)))))
        A, B = A.astype(np.int32), B.astype(np.int32)
        r = dg.spmspm_symbolic(n, A, B)
        off, ln, st = oracle.c_structure(n, A, B)
        assert np.array_equal(r["C_off"], off) and np.array_equal(r["C_len"], ln)
        assert np.array_equal(r["C_start"], st)
        ptr, pa, pb = oracle.pair_lists(n, A, B, off)
        assert np.array_equal(r["pair_ptr"], ptr)
        assert np.array_equal(r["pair_a"], pa) and np.array_equal(r["pair_b"], pb)
