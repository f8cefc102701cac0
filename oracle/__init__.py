"""CPU parity oracle for the B200 DIA library -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` /
``--impl reference`` legs of ``bench.py`` may import this package.  The
library (``diagpu_b200``) never imports it and has no CPU path of its own.

``liboracle.so`` is ``dia_oracle.c``: a C restatement of the reference's CPU
routines (each function cites the reference file:line it follows).  The
``_ref/`` shared objects are the reference's own sources compiled by
``oracle/Makefile``; they exist wherever the reference was present at build
time and are used to pin the restatement and, on the GPU box, as the timed
reference CPU baseline.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))

_i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
_i64p = np.ctypeslib.ndpointer(np.int64, flags="C_CONTIGUOUS")
_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_f64p = np.ctypeslib.ndpointer(np.float64, flags="C_CONTIGUOUS")
_lib = None
_ref = {}


def lib():
    """Load liboracle.so (built by ``make -C oracle``)."""
    global _lib
    if _lib is None:
        path = os.path.join(HERE, "liboracle.so")
        if not os.path.exists(path):
            raise RuntimeError(f"oracle not built: {path} missing (run make -C oracle)")
        L = C.CDLL(path)
        i, i64, f, p = C.c_int, C.c_int64, C.c_float, C.c_void_p
        L.orc_build_recon.argtypes = [i, i, i, _i32p, _i32p, _i32p, _f32p, _i32p, _f32p]
        L.orc_spmv_recon.argtypes = [i, i, i, _i32p, _f32p, _f32p, i, _f32p]
        L.orc_spmv_csr.argtypes = [i, _i32p, _i32p, _f32p, _f32p, _f32p]
        L.orc_spmv_rowidx.argtypes = [i64, i64, i64, i, _i32p, _f32p, i64, _f32p, i64, i64, _f32p, i]
        L.orc_expm_taylor.argtypes = [i64, i, _i32p, _f32p, i64, f, i, _f32p, _f32p, i]
        L.orc_lanczos.argtypes = [i64, i, _i32p, _f32p, i64, i, _f32p, _f64p, _f64p, p]
        L.orc_spmv_rowidx_c64.argtypes = [i64, i64, i, _i32p, _f32p, i64, _f32p, _f32p, i]
        L.orc_expm_taylor_c64.argtypes = [i64, i, _i32p, _f32p, i64, f, i, _f32p, _f32p, i]
        L.orc_c_structure.argtypes = [i, _i32p, i, _i32p, i, p, p, p]
        L.orc_c_structure.restype = i
        L.orc_pair_lists.argtypes = [i, _i32p, i, _i32p, i, _i32p, i, p, p, p]
        L.orc_pair_lists.restype = i64
        hm = [_i32p, _i32p, _i64p, _f32p, i]
        L.orc_dia_spgemm_hm.argtypes = [i] + hm + hm + [_i32p, _i32p, _i64p, i, _f32p, i]
        L.orc_dia_spgemm_hm_f64.argtypes = [i] + hm + hm + [_i32p, _i32p, _i64p, i, _f64p, i]
        L.orc_build_c_layout.argtypes = [i, _i32p, i, _i32p, i, p, p, p, p, p]
        L.orc_build_c_layout.restype = i
        L.orc_gemm_diag_f32.argtypes = [_f32p, _i32p, i, _f32p, _i32p, i, i, _f32p, _i32p, _i32p]
        L.orc_gemm_diag_f64.argtypes = [_f32p, _i32p, i, _f32p, _i32p, i, i, _f64p, _i32p, _i32p, i]
        L.orc_synth_rowidx.argtypes = [C.c_uint64, i64, i64, i, _i32p, p, i, f, f, i64, i64, i64, _f32p]
        L.orc_synth_vector.argtypes = [C.c_uint64, i64, i64, f, f, _f32p]
        _lib = L
    return _lib


def threads() -> int:
    return max(1, os.cpu_count() or 1)


def _a(x, dt):
    return np.ascontiguousarray(x, dtype=dt)


def _ptr(x):
    return None if x is None else x.ctypes.data_as(C.c_void_p)


# --------------------------------------------------------------------- SpMV

def build_recon(rows, cols, offsets, starts, lengths, values):
    """DIA storage -> (descending offsets, K x cols Recon)."""
    K = len(offsets)
    off = np.empty(K, np.int32)
    rec = np.empty(K * cols, np.float32)
    lib().orc_build_recon(rows, cols, K, _a(offsets, np.int32), _a(starts, np.int32),
                          _a(lengths, np.int32), _a(values, np.float32), off, rec)
    return off, rec.reshape(K, cols)


def spmv_recon(rows, cols, offsets, recon, x, x_size=None):
    y = np.empty(rows, np.float32)
    x = _a(x, np.float32)
    lib().orc_spmv_recon(rows, cols, len(offsets), _a(offsets, np.int32),
                         _a(recon, np.float32).reshape(-1), x,
                         int(cols if x_size is None else x_size), y)
    return y


def spmv_csr(n, rowptr, colidx, vals, x):
    y = np.empty(n, np.float32)
    lib().orc_spmv_csr(n, _a(rowptr, np.int32), _a(colidx, np.int32), _a(vals, np.float32),
                       _a(x, np.float32), y)
    return y


def spmv_rowidx(offsets, vals, stride, x, *, ncols, row0=0, nrows=None, x_lo=0, nthreads=None):
    """y for rows [row0, row0+nrows) of a padded row-indexed matrix."""
    K = len(offsets)
    vals = _a(vals, np.float32).reshape(-1)
    if nrows is None:
        nrows = vals.size // K if K else 0
        nrows = min(nrows, stride)
    y = np.empty(nrows, np.float32)
    x = _a(x, np.float32)
    lib().orc_spmv_rowidx(row0, nrows, ncols, K, _a(offsets, np.int32), vals, stride, x,
                          x_lo, x.size, y, nthreads or threads())
    return y


def expm_taylor(offsets, vals, stride, t, m, x, *, nthreads=None):
    """y = sum_{j<=m} (tA)^j x / j! by the recurrence of orc_expm_taylor."""
    x = _a(x, np.float32)
    y = np.empty(x.size, np.float32)
    lib().orc_expm_taylor(x.size, len(offsets), _a(offsets, np.int32),
                          _a(vals, np.float32).reshape(-1), stride, float(t), int(m), x, y,
                          nthreads or threads())
    return y


def lanczos(offsets, vals, stride, m, x, *, basis=False):
    """(alpha, beta[, basis]) of m Lanczos steps by orc_lanczos."""
    x = _a(x, np.float32)
    al = np.zeros(max(m, 1), np.float64)
    be = np.zeros(max(m, 1), np.float64)
    B = np.zeros((max(m, 1), x.size), np.float32) if basis else None
    lib().orc_lanczos(x.size, len(offsets), _a(offsets, np.int32), _a(vals, np.float32).reshape(-1),
                      stride, int(m), x, al, be, B.ctypes.data_as(C.c_void_p) if basis else None)
    return (al[:m], be[:m], B[:m]) if basis else (al[:m], be[:m])


def _c64_as_f32(a):
    a = np.ascontiguousarray(a, np.complex64)
    return a.view(np.float32).reshape(-1)


def spmv_c64(offsets, vals, stride, x, *, n_rows, n_cols, nthreads=None):
    """y = A x for complex64 A (rows layout [K, stride]) and x."""
    y = np.empty(2 * n_rows, np.float32)
    lib().orc_spmv_rowidx_c64(n_rows, n_cols, len(offsets), _a(offsets, np.int32),
                              _c64_as_f32(vals), stride, _c64_as_f32(x), y, nthreads or threads())
    return y.view(np.complex64)


def expm_taylor_c64(offsets, vals, stride, t, m, x, *, nthreads=None):
    """exp(-i t A) x by the truncated Taylor recurrence of orc_expm_taylor_c64."""
    x = np.ascontiguousarray(x, np.complex64)
    y = np.empty(2 * x.size, np.float32)
    lib().orc_expm_taylor_c64(x.size, len(offsets), _a(offsets, np.int32), _c64_as_f32(vals),
                              stride, float(t), int(m), _c64_as_f32(x), y, nthreads or threads())
    return y.view(np.complex64)


# ------------------------------------------------------------ SpMSpM symbolic

def c_structure(n, A_off, B_off):
    """(offsets, lengths, starts) of C = A*B (make_c_structure)."""
    A_off = _a(A_off, np.int32)
    B_off = _a(B_off, np.int32)
    nC = lib().orc_c_structure(n, A_off, len(A_off), B_off, len(B_off), None, None, None)
    off = np.empty(nC, np.int32)
    ln = np.empty(nC, np.int32)
    st = np.empty(nC, np.int64)
    lib().orc_c_structure(n, A_off, len(A_off), B_off, len(B_off), _ptr(off), _ptr(ln), _ptr(st))
    return off, ln, st


def pair_lists(n, A_off, B_off, C_off):
    A_off, B_off, C_off = (_a(v, np.int32) for v in (A_off, B_off, C_off))
    np_ = lib().orc_pair_lists(n, A_off, len(A_off), B_off, len(B_off), C_off, len(C_off),
                               None, None, None)
    ptr = np.empty(len(C_off) + 1, np.int32)
    pa = np.empty(max(np_, 1), np.int32)
    pb = np.empty(max(np_, 1), np.int32)
    lib().orc_pair_lists(n, A_off, len(A_off), B_off, len(B_off), C_off, len(C_off),
                         _ptr(ptr), _ptr(pa), _ptr(pb))
    return ptr, pa[:np_], pb[:np_]


# ------------------------------------------------------------- SpMSpM numeric

def hm_starts(n, off):
    ln = (n - np.abs(_a(off, np.int64))).astype(np.int32)
    st = np.zeros(len(ln), np.int64)
    if len(ln):
        st[1:] = np.cumsum(ln[:-1], dtype=np.int64)
    return ln, st


def dia_spgemm_hm(n, A, B, C_struct, *, f64=False, nthreads=None):
    """C = A*B on HM arrays.  A/B = (off, len, start, vals); C_struct =
    (off, len, start).  Returns the flat C values."""
    Ao, Al, As, Av = A
    Bo, Bl, Bs, Bv = B
    Co, Cl, Cs = C_struct
    nnz = int(Cs[-1] + Cl[-1]) if len(Cl) else 0
    args = [n, _a(Ao, np.int32), _a(Al, np.int32), _a(As, np.int64), _a(Av, np.float32), len(Ao),
            _a(Bo, np.int32), _a(Bl, np.int32), _a(Bs, np.int64), _a(Bv, np.float32), len(Bo),
            _a(Co, np.int32), _a(Cl, np.int32), _a(Cs, np.int64), len(Co)]
    if f64:
        out = np.zeros(nnz, np.float64)
        lib().orc_dia_spgemm_hm_f64(*args, out, nthreads or threads())
    else:
        out = np.zeros(nnz, np.float32)
        lib().orc_dia_spgemm_hm(*args, out, nthreads or threads())
    return out


# ------------------------------------------------------------------ gemm_diag

def build_c_layout(n, off_A, off_B):
    off_A = _a(off_A, np.int32)
    off_B = _a(off_B, np.int32)
    L = lib()
    tot = C.c_int64(0)
    nk = L.orc_build_c_layout(n, off_A, len(off_A), off_B, len(off_B), None, None, None, None,
                              C.byref(tot))
    co = np.empty(nk, np.int32)
    cl = np.empty(nk, np.int32)
    k2i = np.empty(2 * n - 1, np.int32)
    kl = np.empty(nk, np.int32)
    L.orc_build_c_layout(n, off_A, len(off_A), off_B, len(off_B), _ptr(co), _ptr(cl), _ptr(k2i),
                         _ptr(kl), C.byref(tot))
    return co, cl, k2i, kl, int(tot.value)


def gemm_diag(DA, off_A, DB, off_B, n, *, f64=True, nthreads=None):
    """Row-packed DA/DB (P x n, Q x n) -> HM-packed C (values, layout)."""
    co, cl, k2i, kl, tot = build_c_layout(n, off_A, off_B)
    DA = _a(DA, np.float32).reshape(-1)
    DB = _a(DB, np.float32).reshape(-1)
    oA = _a(off_A, np.int32)
    oB = _a(off_B, np.int32)
    if f64:
        out = np.zeros(tot, np.float64)
        lib().orc_gemm_diag_f64(DA, oA, len(oA), DB, oB, len(oB), n, out, co, k2i,
                                nthreads or threads())
    else:
        out = np.zeros(tot, np.float32)
        lib().orc_gemm_diag_f32(DA, oA, len(oA), DB, oB, len(oB), n, out, co, k2i)
    return out, (co, cl, k2i, kl, tot)


# ------------------------------------------------------------------ synthetic

def synth_rowidx(seed, n_rows, n_cols, offsets, *, kind=0, lo=-1.0, hi=1.0, base=None,
                 row0=0, nrows=None, stride=None):
    offsets = _a(offsets, np.int32)
    if nrows is None:
        nrows = n_rows - row0
    if stride is None:
        stride = (nrows + 31) // 32 * 32
    vals = np.empty(len(offsets) * stride, np.float32)
    b = None if base is None else _a(base, np.float32)
    lib().orc_synth_rowidx(seed, n_rows, n_cols, len(offsets), offsets, _ptr(b), kind, lo, hi,
                           row0, nrows, stride, vals)
    return vals.reshape(len(offsets), stride)


def synth_vector(seed, n, *, lo=-1.0, hi=1.0, i0=0):
    out = np.empty(n, np.float32)
    lib().orc_synth_vector(seed, i0, n, lo, hi, out)
    return out


# ------------------------------------------------------ reference (compiled)

def ref(name):
    """ctypes handle of oracle/_ref/libref_<name>.so, or None when absent."""
    if name not in _ref:
        path = os.path.join(HERE, "_ref", f"libref_{name}.so")
        _ref[name] = C.CDLL(path) if os.path.exists(path) else None
    return _ref[name]
