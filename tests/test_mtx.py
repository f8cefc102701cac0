"""Matrix Market ingestion (dia_mtx_read, host side: runs without a GPU).

The golden file is the reference's own generator output
(spmv/tools/gen_banded_mtx.cpp, compiled unmodified; see
tests/golden/make_golden.py); scipy.io.mmread is the independent reader the
results are compared with, entry for entry."""
import ctypes as C
import os
import warnings

import numpy as np
import pytest
import scipy.io as sio

import diagpu_b200 as dg

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def _dense_from_rows(n_rows, n_cols, offs, vals):
    A = np.zeros((n_rows, n_cols), np.float32)
    for k, d in enumerate(offs):
        for i in range(n_rows):
            j = i + int(d)
            if 0 <= j < n_cols:
                A[i, j] = vals[k, i]
            else:
                assert vals[k, i] == 0.0          # out-of-matrix entries are zero
        assert (vals[k, n_rows:] == 0.0).all()    # stride padding is zero
    return A


def _scipy_dense(path):
    with warnings.catch_warnings():
        warnings.simplefilter("ignore")
        return np.asarray(sio.mmread(path).toarray(), np.float64).astype(np.float32)


def test_golden_reference_generator_file():
    path = os.path.join(GOLDEN, "banded_64.mtx")
    n_rows, n_cols, offs, vals = dg.read_mtx_host(path)
    assert (n_rows, n_cols) == (64, 64)
    assert np.array_equal(offs, [-9, -5, -2, -1, 0, 1, 2, 5, 9])   # the generator's set
    assert np.array_equal(_dense_from_rows(n_rows, n_cols, offs, vals), _scipy_dense(path))


CASES = {
    "symmetric": ("real symmetric", 5, 5,
                  [(1, 1, 2.5), (3, 1, -1.25), (5, 2, 0.5), (4, 4, 7.0)]),
    "skew": ("real skew-symmetric", 4, 4, [(2, 1, 3.0), (4, 3, -0.75)]),
    "pattern": ("pattern general", 3, 6, [(1, 6), (2, 2), (3, 1)]),
    "integer": ("integer general", 4, 4, [(1, 2, 7), (4, 1, -3), (2, 2, 11)]),
    "duplicates": ("real general", 3, 3, [(1, 1, 0.1), (1, 1, 0.2), (2, 3, 1e-8), (2, 3, 1.0)]),
    "rectangular": ("real general", 3, 7, [(1, 7, 1.5), (3, 1, -2.0), (2, 2, 0.125)]),
}


def _write(path, kind, m, n, entries, comments=True):
    with open(path, "w") as f:
        f.write(f"%%MatrixMarket matrix coordinate {kind}\n")
        if comments:
            f.write("% a comment\n%\n\n")
        f.write(f"{m} {n} {len(entries)}\n")
        for e in entries:
            f.write(" ".join(str(x) for x in e) + "\n")


@pytest.mark.parametrize("case", sorted(CASES))
def test_formats_match_scipy(tmp_path, case):
    kind, m, n, entries = CASES[case]
    path = str(tmp_path / f"{case}.mtx")
    _write(path, kind, m, n, entries)
    n_rows, n_cols, offs, vals = dg.read_mtx_host(path)
    assert (n_rows, n_cols) == (m, n)
    assert np.all(np.diff(offs) > 0)               # ascending, distinct
    assert np.array_equal(_dense_from_rows(n_rows, n_cols, offs, vals), _scipy_dense(path))


@pytest.mark.parametrize("banner,code", [
    ("%%MatrixMarket matrix array real general", dg.DIA_ERR_UNSUPPORTED),
    ("%%MatrixMarket matrix coordinate complex general", dg.DIA_ERR_UNSUPPORTED),
    ("%%MatrixMarket matrix coordinate real hermitian", dg.DIA_ERR_UNSUPPORTED),
    ("%%NotMatrixMarket matrix coordinate real general", dg.DIA_ERR_INVALID),
])
def test_rejected_files(tmp_path, banner, code):
    path = str(tmp_path / "bad.mtx")
    with open(path, "w") as f:
        f.write(banner + "\n2 2 1\n1 1 1.0 0.0\n")
    with pytest.raises(dg.DiaError) as e:
        dg.read_mtx_host(path)
    assert e.value.code == code


def test_malformed_entries(tmp_path):
    for body, name in (("3 3 2\n1 1 1.0\n", "truncated"), ("3 3 1\n4 1 1.0\n", "outside"),
                       ("3 3 1\n1 1\n", "no value"), ("x y z\n", "size line")):
        path = str(tmp_path / "m.mtx")
        with open(path, "w") as f:
            f.write("%%MatrixMarket matrix coordinate real general\n" + body)
        with pytest.raises(dg.DiaError) as e:
            dg.read_mtx_host(path)
        assert e.value.code == dg.DIA_ERR_INVALID, name
    with pytest.raises(dg.DiaError):
        dg.read_mtx_host(str(tmp_path / "missing.mtx"))


def test_capacity_two_call_pattern():
    L = dg.lib()
    path = os.fsencode(os.path.join(GOLDEN, "banded_64.mtx"))
    nr, nc, K = C.c_int64(0), C.c_int64(0), C.c_int(0)
    assert L.dia_mtx_read(path, C.byref(nr), C.byref(nc), C.byref(K), None, None, 0) == 0
    assert K.value == 9
    small = C.c_int(4)
    offs = np.empty(4, np.int32)
    rc = L.dia_mtx_read(path, C.byref(nr), C.byref(nc), C.byref(small),
                        offs.ctypes.data_as(C.c_void_p), None, 0)
    assert rc == dg.DIA_ERR_CAPACITY and small.value == 9


def test_write_then_read_round_trip(tmp_path):
    """DIA -> Matrix Market -> DIA: offsets and every fp32 value come back
    exactly (9 significant digits), stored zeros included."""
    rng = np.random.default_rng(11)
    n_rows, n_cols = 300, 257
    offs = np.array([-120, -7, 0, 3, 200], np.int32)
    stride = 320
    vals = np.zeros((len(offs), stride), np.float32)
    for k, d in enumerate(offs):
        lo, hi = max(0, -d), min(n_rows, n_cols - d)
        vals[k, lo:hi] = rng.standard_normal(hi - lo).astype(np.float32) * 10.0 ** rng.integers(-8, 8)
    vals[2, 5] = 0.0                                   # a stored zero keeps its diagonal
    path = str(tmp_path / "rt.mtx")
    dg.write_mtx(path, n_rows, n_cols, offs, vals)
    r, c, o2, v2 = dg.read_mtx_host(path)
    assert (r, c) == (n_rows, n_cols) and np.array_equal(o2, offs)
    assert np.array_equal(v2[:, :n_rows], vals[:, :n_rows])
    assert np.array_equal(_dense_from_rows(r, c, o2, v2), _scipy_dense(path))


def test_write_reproduces_the_reference_generator_structure(tmp_path):
    """Reading the reference generator's file and writing it again keeps the
    entry order (rows, then offsets ascending) and the values."""
    src = os.path.join(GOLDEN, "banded_64.mtx")
    n_rows, n_cols, offs, vals = dg.read_mtx_host(src)
    out = str(tmp_path / "again.mtx")
    dg.write_mtx(out, n_rows, n_cols, offs, vals)
    body = lambda p: [ln.split()[:2] for ln in open(p) if not ln.startswith("%")][1:]
    assert body(out) == body(src)
    assert np.array_equal(_scipy_dense(out), _scipy_dense(src))


def _dense_from_rows_c64(n_rows, n_cols, offs, vals):
    A = np.zeros((n_rows, n_cols), np.complex64)
    for k, d in enumerate(offs):
        for i in range(n_rows):
            j = i + int(d)
            if 0 <= j < n_cols:
                A[i, j] = vals[k, i]
            else:
                assert vals[k, i] == 0
        assert (vals[k, n_rows:] == 0).all()
    return A


CASES_C64 = {
    "complex general": ("complex general", 4, 5,
                        [(1, 1, 1.5, -2.0), (2, 5, 0.25, 3.0), (4, 2, -1.0, 0.0), (1, 1, 0.5, 1.0)]),
    "complex hermitian": ("complex hermitian", 4, 4,
                          [(1, 1, 2.0, 0.0), (3, 1, 1.0, -0.5), (4, 2, -0.25, 2.0), (4, 4, 1.0, 0.0)]),
    "complex symmetric": ("complex symmetric", 3, 3, [(2, 1, 1.0, 2.0), (3, 3, -1.0, 0.5)]),
    "complex skew": ("complex skew-symmetric", 3, 3, [(3, 1, 0.5, -1.5)]),
    "real as c64": ("real symmetric", 5, 5, [(1, 1, 2.5), (3, 1, -1.25), (5, 2, 0.5)]),
}


@pytest.mark.parametrize("case", sorted(CASES_C64))
def test_c64_formats_match_scipy(tmp_path, case):
    """dia_mtx_read_c64 against scipy.io.mmread, entry for entry (Hermitian
    files mirror the conjugate, skew-symmetric the negation)."""
    kind, m, n, entries = CASES_C64[case]
    path = str(tmp_path / "c.mtx")
    _write(path, kind, m, n, entries)
    n_rows, n_cols, offs, vals, is_cx = dg.read_mtx_c64_host(path)
    assert (n_rows, n_cols) == (m, n) and is_cx == kind.startswith("complex")
    assert vals.dtype == np.complex64 and np.all(np.diff(offs) > 0)
    with warnings.catch_warnings():
        warnings.simplefilter("ignore")
        ref = np.asarray(sio.mmread(path).toarray(), np.complex128).astype(np.complex64)
    assert np.array_equal(_dense_from_rows_c64(n_rows, n_cols, offs, vals), ref)


def test_c64_real_file_equals_fp32_reader():
    path = os.path.join(GOLDEN, "banded_64.mtx")
    _, _, offs, vals = dg.read_mtx_host(path)
    _, _, o2, v2, is_cx = dg.read_mtx_c64_host(path)
    assert not is_cx and np.array_equal(offs, o2)
    assert np.array_equal(v2.real, vals) and not v2.imag.any()


def test_c64_missing_imaginary_part(tmp_path):
    path = str(tmp_path / "m.mtx")
    with open(path, "w") as f:
        f.write("%%MatrixMarket matrix coordinate complex general\n2 2 1\n1 1 1.0\n")
    with pytest.raises(dg.DiaError) as e:
        dg.read_mtx_c64_host(path)
    assert e.value.code == dg.DIA_ERR_INVALID
