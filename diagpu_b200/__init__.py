"""diagpu_b200 -- B200-native DIA sparse linear algebra (host side).

The compute lives in ``libdiagpu_b200.so`` (CUDA for sm_100a, C ABI declared
in ``include/diagpu_b200.h``).  This module binds that ABI with ctypes and
exposes it on torch CUDA tensors; torch is used only for device memory and
streams.  There is no CPU implementation here: every function raises if the
library is missing or the tensors are not on a CUDA device.

Entry points mirror the reference's launch surfaces:
  spmv_recon        launch_tc_spmv_regdirect (spmv/src/dia_reconstruct.cuh:139-144)
  spmv              CPU CSR loop semantics on the padded rows layout
                    (spmv/bench/bench_cusparse.cu:119-126)
  spmspm_symbolic   make_c_structure + pair lists (spmspm/bench_spmspm.cu:109-243)
  spmspm_hm         gather_meta_kernel argument set (spmspm/spmspm.cu:256-319)
  spmspm            the same product on the padded rows layout
  gemm_diag         gemm_diag_kernel argument set (gemm_diag/gemm_diag.cu:119-131)
"""
from __future__ import annotations

import ctypes as C
import os
from dataclasses import dataclass

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libdiagpu_b200.so")

DIA_OK, DIA_ERR_INVALID, DIA_ERR_CUDA, DIA_ERR_UNSUPPORTED, DIA_ERR_CAPACITY, DIA_ERR_TIMEOUT = range(6)
DIA_TC_TIMEOUT = 1   # dia_device_status bit: a tcgen05 kernel wait ran out
GEMM_AUTO, GEMM_SIMT, GEMM_TCGEN05 = 0, 1, 2
ALIGN = 32  # floats per stride unit (128 bytes)

_lib = None


class DiaError(RuntimeError):
    def __init__(self, code, msg):
        super().__init__(f"[{code}] {msg}")
        self.code = code


def lib():
    """The loaded CUDA library (raises if it was not built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise DiaError(DIA_ERR_UNSUPPORTED,
                           f"{LIB_PATH} missing: build it with __graft_entry__.build()")
        L = C.CDLL(LIB_PATH)
        i, i64, u64, f, p = C.c_int, C.c_int64, C.c_uint64, C.c_float, C.c_void_p
        L.dia_last_error.restype = C.c_char_p
        L.dia_version.restype = i
        L.dia_spmv_recon.argtypes = [i, i, i, p, p, p, i, p, p]
        L.dia_spmv_rows.argtypes = [i64, i64, i, p, p, i64, i64, i64, i64, p, i64, i64, p, p]
        L.dia_spmspm_symbolic.argtypes = [i, p, i, p, i, p, p, p, p, p, p, p, p]
        L.dia_spmspm_hm.argtypes = [p, p, p, p, i, p, p, p, p, p, p, p, p, i, i, p]
        L.dia_spmspm_hm_noalloc.argtypes = [p, p, p, p, i, p, p, p, p, p, p, p, p, i, i, p]
        L.dia_spmspm_rows.argtypes = [i64, p, i64, p, i, p, i64, i64, i64, i64, p, i, p, i64,
                                      p, i, i64, i64, i64, p]
        L.dia_gemm_diag.argtypes = [p, p, p, p, i, i, i, p, p, p, p, p]
        L.dia_gemm_diag_ex.argtypes = [p, p, p, p, p, p, i, i, i, p, p, p, p, i, i, p]
        L.dia_spmspm_plan_create.argtypes = [i64, p, i, p, i, i64, i64, i64, i64, i64, i64, i64,
                                             i64, p]
        L.dia_spmspm_plan_info.argtypes = [p, p, p, p, p, p, p, p]
        L.dia_spmspm_plan_execute.argtypes = [p, p, p, p, i64, i64, i, p]
        L.dia_spmspm_plan_destroy.argtypes = [p]
        for name in ("dia_spmspm_plan_create", "dia_spmspm_plan_info", "dia_spmspm_plan_execute",
                     "dia_spmspm_plan_destroy"):
            getattr(L, name).restype = i
        L.dia_nccl_unique_id.argtypes = [p, i]
        L.dia_dist_create.argtypes = [i, i, p, p]
        L.dia_dist_create_timeout.argtypes = [i, i, p, i64, p]
        L.dia_dist_abort.argtypes = [p]
        L.dia_dist_halo_start.argtypes = [p, p, i64, i64, i, p, p]
        L.dia_dist_halo_wait.argtypes = [p, p]
        L.dia_dist_spmv_step.argtypes = [p, i64, i64, i, p, p, i64, i64, p, i64, i64, p, p, i64,
                                         i64, i64, i64, i, p]
        L.dia_dist_async_error.argtypes = [p]
        L.dia_dist_destroy.argtypes = [p]
        L.dia_spmv_rows_peer.argtypes = [p, u64, i64, i64, i, p, p, i64, i64, i64, i64, i64, i64,
                                         i, i, p, p, p]
        L.dia_dist_peer_setup.argtypes = [p, i64, i64, i64, i64, p]
        L.dia_dist_spmv_fused.argtypes = [p, i64, i64, i, p, p, i64, i64, i, i, p, p, p]
        L.dia_dist_set_timeout.argtypes = [p, i64]
        L.dia_dist_status.argtypes = [p, p, i]
        for name in ("dia_nccl_unique_id", "dia_dist_create", "dia_dist_halo_start",
                     "dia_dist_halo_wait", "dia_dist_spmv_step", "dia_dist_async_error",
                     "dia_dist_destroy", "dia_dist_create_timeout", "dia_dist_abort",
                     "dia_spmv_rows_peer", "dia_dist_peer_setup",
                     "dia_dist_spmv_fused", "dia_dist_set_timeout", "dia_dist_status"):
            getattr(L, name).restype = i
        L.dia_device_status.argtypes = [p, i]
        L.dia_device_status.restype = i
        L.dia_test_tc_wait.argtypes = [u64, i]
        L.dia_test_tc_wait.restype = i
        L.dia_synth_rows.argtypes = [u64, i64, i64, i, p, p, i, f, f, i64, i64, i64, p, p]
        L.dia_synth_vector.argtypes = [u64, i64, i64, f, f, p, p]
        L.dia_lanczos_workspace.argtypes = [i64]
        L.dia_lanczos_workspace.restype = i64
        L.dia_lanczos.argtypes = [i64, i, p, p, i64, i, p, p, p, p, p, i64, p]
        L.dia_lanczos.restype = i
        L.dia_spmv_rows_c64.argtypes = [i64, i64, i, p, p, i64, p, p, p]
        L.dia_expm_taylor_c64.argtypes = [i64, i, p, p, i64, f, i, p, p, p, p]
        for name in ("dia_spmv_rows_c64", "dia_expm_taylor_c64"):
            getattr(L, name).restype = i
        L.dia_pauli_to_dia.argtypes = [i, i, p, p, p, p, p, p, p, i64, p]
        L.dia_pauli_to_dia.restype = i
        L.dia_mtx_read.argtypes = [C.c_char_p, p, p, p, p, p, i64]
        L.dia_mtx_write.argtypes = [C.c_char_p, i64, i64, i, p, p, i64]
        L.dia_mtx_write.restype = i
        L.dia_mtx_read.restype = i
        L.dia_mtx_read_c64.argtypes = [C.c_char_p, p, p, p, p, p, i64, p]
        L.dia_mtx_read_c64.restype = i
        L.dia_expm_taylor.argtypes = [i64, i, p, p, i64, f, i, p, p, p, p]
        L.dia_expm_taylor.restype = i
        L.dia_spmspm_device_workspace.argtypes = [i64, i, i, i]
        L.dia_spmspm_device_workspace.restype = i64
        L.dia_spmspm_symbolic_device.argtypes = [i64, p, p, i, p, i, p, p, i, p, i64, p]
        L.dia_spmspm_rows_device.argtypes = [i64, p, p, i, p, i64, p, i, p, i64, p, p, i, p,
                                             i64, p, i64, p]
        for name in ("dia_spmspm_symbolic_device", "dia_spmspm_rows_device"):
            getattr(L, name).restype = i
        for name in ("dia_spmv_recon", "dia_spmv_rows", "dia_spmspm_symbolic", "dia_spmspm_hm",
                     "dia_spmspm_hm_noalloc", "dia_spmspm_rows", "dia_gemm_diag", "dia_gemm_diag_ex", "dia_synth_rows",
                     "dia_synth_vector"):
            getattr(L, name).restype = i
        _lib = L
    return _lib


def check(rc):
    if rc != DIA_OK:
        raise DiaError(rc, lib().dia_last_error().decode())


def _stream(stream=None):
    s = stream if stream is not None else torch.cuda.current_stream()
    return C.c_void_p(s.cuda_stream)


def _dptr(t, dtype=None):
    if t is None:
        return None
    if not t.is_cuda:
        raise DiaError(DIA_ERR_INVALID, "tensor must be on a CUDA device")
    if dtype is not None and t.dtype != dtype:
        raise DiaError(DIA_ERR_INVALID, f"expected {dtype}, got {t.dtype}")
    if not t.is_contiguous():
        raise DiaError(DIA_ERR_INVALID, "tensor must be contiguous")
    return C.c_void_p(t.data_ptr())


def round_stride(rows: int) -> int:
    """Diagonal stride in floats: rows rounded up to 32 (128-byte rows).
    When that is a multiple of 2048 floats, 64 floats are added: diagonals a
    large power of two apart keep the same low address bits, so the many
    diagonal streams of a product land on the same HBM channels (measured
    on config 5 C = A*A: 24-27 ms unpadded, 21-22 ms padded)."""
    s = (rows + ALIGN - 1) // ALIGN * ALIGN
    return s + 64 if s % 2048 == 0 else s


# ------------------------------------------------------------------ storage

@dataclass
class DiaRows:
    """A row block of an n_rows x n_cols DIA matrix in the padded rows layout.

    vals[k, i - vrow0] = A[i, i + offsets[k]] for global rows
    i in [vrow0, vrow0 + nrows); zero where the column leaves [0, n_cols) and
    in the stride padding.  A whole matrix is the block with vrow0 = 0,
    nrows = n_rows.
    """
    n_rows: int
    n_cols: int
    offsets: np.ndarray      # host int32 [K]
    d_offsets: torch.Tensor  # device int32 [K]
    vals: torch.Tensor       # device float32 [K, stride]
    vrow0: int = 0
    nrows: int | None = None

    def __post_init__(self):
        if self.nrows is None:
            self.nrows = self.n_rows - self.vrow0

    @property
    def K(self):
        return len(self.offsets)

    @property
    def stride(self):
        return self.vals.shape[1]

    @property
    def nnz(self):
        """Stored (in-range) entries of this block's rows."""
        r0, r1 = self.vrow0, self.vrow0 + self.nrows
        return int(sum(max(0, min(r1, self.n_cols - int(d)) - max(r0, -int(d)))
                       for d in self.offsets))

    @property
    def max_abs_offset(self):
        return int(np.abs(self.offsets).max()) if self.K else 0

    @staticmethod
    def empty(n_rows, n_cols, offsets, *, vrow0=0, nrows=None, device="cuda", zero=True,
              dtype=torch.float32):
        """dtype float32, or complex64 for the complex paths (spmv_c64,
        expm_taylor_c64; stride then counts complex elements)."""
        offsets = np.ascontiguousarray(offsets, np.int32)
        nrows = n_rows - vrow0 if nrows is None else nrows
        alloc = torch.zeros if zero else torch.empty
        vals = alloc((len(offsets), round_stride(nrows)), dtype=dtype, device=device)
        d_off = torch.from_numpy(offsets.copy()).to(device)
        return DiaRows(n_rows, n_cols, offsets, d_off, vals, vrow0, nrows)

    @staticmethod
    def synth(n_rows, n_cols, offsets, seed, *, kind=0, lo=-1.0, hi=1.0, base=None, vrow0=0,
              nrows=None, device="cuda", stream=None):
        """Generate a row block with the library's counter-based generator
        (value depends only on seed, offset and global row)."""
        A = DiaRows.empty(n_rows, n_cols, offsets, vrow0=vrow0, nrows=nrows, device=device,
                          zero=False)
        d_base = None
        if base is not None:
            d_base = torch.as_tensor(np.asarray(base, np.float32), device=device)
        with torch.cuda.device(A.vals.device):
            check(lib().dia_synth_rows(seed, n_rows, n_cols, A.K, _dptr(A.d_offsets),
                                       _dptr(d_base), kind, lo, hi, vrow0, A.nrows, A.stride,
                                       _dptr(A.vals), _stream(stream)))
        return A

    @staticmethod
    def from_host(n_rows, n_cols, offsets, vals_rows, *, vrow0=0, device="cuda"):
        """From a host [K, nrows] array in rows layout (no padding needed);
        a complex array gives a complex64 matrix."""
        cplx = np.iscomplexobj(vals_rows)
        vals_rows = np.asarray(vals_rows, np.complex64 if cplx else np.float32)
        A = DiaRows.empty(n_rows, n_cols, offsets, vrow0=vrow0, nrows=vals_rows.shape[1],
                          device=device, dtype=torch.complex64 if cplx else torch.float32)
        A.vals[:, :vals_rows.shape[1]] = torch.from_numpy(vals_rows).to(device)
        return A

    def to_host_rows(self):
        return self.vals[:, :self.nrows].cpu().numpy()


def synth_vector(n, seed, *, lo=-1.0, hi=1.0, i0=0, device="cuda", out=None, stream=None):
    out = torch.empty(n, dtype=torch.float32, device=device) if out is None else out
    with torch.cuda.device(out.device):
        check(lib().dia_synth_vector(seed, i0, n, lo, hi, _dptr(out), _stream(stream)))
    return out


# --------------------------------------------------------------------- SpMV

def spmv_recon(rows, cols, d_offsets, d_values, x, y=None, x_size=None, stream=None):
    """y = A*x for the reference's ReconView (column-indexed, K x cols)."""
    y = torch.empty(rows, dtype=torch.float32, device=x.device) if y is None else y
    xs = x.numel() if x_size is None else x_size
    check(lib().dia_spmv_recon(rows, cols, d_offsets.numel(), _dptr(d_offsets, torch.int32),
                               _dptr(d_values, torch.float32), _dptr(x, torch.float32), xs,
                               _dptr(y, torch.float32), _stream(stream)))
    return y


def spmv(A: DiaRows, x, y=None, *, x_lo=0, row_lo=None, row_hi=None, stream=None):
    """y = A*x over the block's rows (or [row_lo, row_hi)).  x holds global
    columns [x_lo, x_lo + len(x)); y is indexed from the block's first row."""
    y = torch.empty(A.stride, dtype=torch.float32, device=A.vals.device) if y is None else y
    lo = A.vrow0 if row_lo is None else row_lo
    hi = A.vrow0 + A.nrows if row_hi is None else row_hi
    check(lib().dia_spmv_rows(A.n_rows, A.n_cols, A.K, _dptr(A.d_offsets), _dptr(A.vals),
                              A.stride, A.vrow0, lo, hi, _dptr(x, torch.float32), x_lo,
                              x_lo + x.numel(), _dptr(y, torch.float32), _stream(stream)))
    return y


# ------------------------------------------------------------------- SpMSpM

def spmspm_symbolic(n, A_off, B_off):
    """Output structure and pair lists of C = A*B (host, exact)."""
    A_off = np.ascontiguousarray(A_off, np.int32)
    B_off = np.ascontiguousarray(B_off, np.int32)
    L = lib()
    nc = C.c_int(0)
    npairs = C.c_int64(0)
    pa = lambda a: a.ctypes.data_as(C.c_void_p)
    check(L.dia_spmspm_symbolic(n, pa(A_off), len(A_off), pa(B_off), len(B_off), C.byref(nc),
                                None, None, None, C.byref(npairs), None, None, None))
    C_off = np.empty(nc.value, np.int32)
    C_len = np.empty(nc.value, np.int32)
    C_start = np.empty(nc.value, np.int64)
    ptr = np.empty(nc.value + 1, np.int32)
    pair_a = np.empty(max(npairs.value, 1), np.int32)
    pair_b = np.empty(max(npairs.value, 1), np.int32)
    check(L.dia_spmspm_symbolic(n, pa(A_off), len(A_off), pa(B_off), len(B_off), C.byref(nc),
                                pa(C_off), pa(C_len), pa(C_start), C.byref(npairs), pa(ptr),
                                pa(pair_a), pa(pair_b)))
    return dict(C_off=C_off, C_len=C_len, C_start=C_start, pair_ptr=ptr,
                pair_a=pair_a[:npairs.value], pair_b=pair_b[:npairs.value])


def spmspm_hm(A_values, A_starts, A_off, A_len, B_values, B_starts, B_len, B_lookup, C_values,
              C_starts, C_off, C_len, n, stream=None):
    """C = A*B with gather_meta_kernel's arguments (device tensors; starts int64)."""
    check(lib().dia_spmspm_hm(_dptr(A_values, torch.float32), _dptr(A_starts, torch.int64),
                              _dptr(A_off, torch.int32), _dptr(A_len, torch.int32),
                              A_off.numel(), _dptr(B_values, torch.float32),
                              _dptr(B_starts, torch.int64), _dptr(B_len, torch.int32),
                              _dptr(B_lookup, torch.int32), _dptr(C_values, torch.float32),
                              _dptr(C_starts, torch.int64), _dptr(C_off, torch.int32),
                              _dptr(C_len, torch.int32), C_off.numel(), n, _stream(stream)))
    return C_values


def lanczos(A: DiaRows, m, x, *, basis=False, stream=None):
    """m Lanczos steps on a symmetric whole matrix (dia_lanczos), all on the
    device.  Returns device fp64 tensors (alpha [m], beta [m]) of the
    tridiagonal T_m, and with basis=True also the fp32 Lanczos vectors
    [m, n]; eigenvalues of T_m (e.g. numpy.linalg.eigvalsh) approach A's
    extreme eigenvalues.  Nothing synchronises with the host."""
    if A.vrow0 != 0 or A.nrows != A.n_rows or A.n_rows != A.n_cols:
        raise DiaError(DIA_ERR_INVALID, "lanczos: A must be a whole square matrix")
    n = A.n_rows
    dev = x.device
    alpha = torch.zeros(max(m, 1), dtype=torch.float64, device=dev)
    beta = torch.zeros(max(m, 1), dtype=torch.float64, device=dev)
    B = torch.empty((max(m, 1), n), dtype=torch.float32, device=dev) if basis else None
    L = lib()
    ws = L.dia_lanczos_workspace(n)
    work = torch.empty(max(ws, 1), dtype=torch.uint8, device=dev)
    with torch.cuda.device(dev):
        check(L.dia_lanczos(n, A.K, _dptr(A.d_offsets), _dptr(A.vals), A.stride, int(m),
                            _dptr(x, torch.float32), _dptr(alpha), _dptr(beta), _dptr(B),
                            _dptr(work), ws, _stream(stream)))
    out = (alpha[:m], beta[:m])
    return out + (B[:m],) if basis else out


def _whole_c64(A, who):
    if A.vals.dtype != torch.complex64:
        raise DiaError(DIA_ERR_INVALID, f"{who}: A must hold complex64 values")
    if A.vrow0 != 0 or A.nrows != A.n_rows:
        raise DiaError(DIA_ERR_INVALID, f"{who}: A must be a whole matrix")


def spmv_c64(A: DiaRows, x, y=None, *, stream=None):
    """y = A x for a complex64 matrix and vector (dia_spmv_rows_c64)."""
    _whole_c64(A, "spmv_c64")
    y = torch.empty(A.n_rows, dtype=torch.complex64, device=x.device) if y is None else y
    with torch.cuda.device(x.device):
        check(lib().dia_spmv_rows_c64(A.n_rows, A.n_cols, A.K, _dptr(A.d_offsets), _dptr(A.vals),
                                      A.stride, _dptr(x, torch.complex64),
                                      _dptr(y, torch.complex64), _stream(stream)))
    return y


def expm_taylor_c64(A: DiaRows, t, m, x, y=None, *, work=None, stream=None):
    """y = exp(-i t A) x by the truncated Taylor series of m terms
    (dia_expm_taylor_c64), e.g. the time evolution of a Hamiltonian."""
    _whole_c64(A, "expm_taylor_c64")
    if A.n_rows != A.n_cols:
        raise DiaError(DIA_ERR_INVALID, "expm_taylor_c64: A must be square")
    n = A.n_rows
    y = torch.empty(n, dtype=torch.complex64, device=x.device) if y is None else y
    work = torch.empty(2 * n, dtype=torch.complex64, device=x.device) if work is None else work
    with torch.cuda.device(x.device):
        check(lib().dia_expm_taylor_c64(n, A.K, _dptr(A.d_offsets), _dptr(A.vals), A.stride,
                                        float(t), int(m), _dptr(x, torch.complex64),
                                        _dptr(y, torch.complex64),
                                        _dptr(work, torch.complex64), _stream(stream)))
    return y


def parse_pauli_sum(text):
    """Terms of a Pauli-string sum in OpenFermion's QubitOperator text form,
    e.g. "0.5 [X0 Y1] +\n(-0.25+0.1j) [Z2] +\n1.0 []"  ->  [(coef, "X0 Y1"), ...]."""
    import re
    terms = []
    for m in re.finditer(r"([^\[\]]*)\[([^\]]*)\]", text):
        coef = m.group(1).strip()
        coef = re.sub(r"^\+", "", coef).strip()
        coef = coef.replace(" ", "")
        terms.append((complex(coef) if coef else 1.0, m.group(2).strip()))
    return terms


def _pauli_masks(terms, nq, big_endian):
    xs, zs, cre, cim = [], [], [], []
    top = 0
    for coef, ops in terms:
        x = z = 0
        for op in ops.split():
            p_, q = op[0].upper(), int(op[1:])
            top = max(top, q + 1)
            if nq is not None and q >= nq:
                raise DiaError(DIA_ERR_INVALID, f"pauli_to_dia: qubit {q} >= nq = {nq}")
            b = (nq - 1 - q) if big_endian else q
            if p_ in "XY":
                x |= 1 << b
            if p_ in "ZY":
                z |= 1 << b
            if p_ not in "XYZI":
                raise DiaError(DIA_ERR_INVALID, f"pauli_to_dia: unknown operator {op!r}")
        xs.append(x)
        zs.append(z)
        c = complex(coef)
        cre.append(c.real)
        cim.append(c.imag)
    return (np.array(xs, np.uint64), np.array(zs, np.uint64), np.array(cre, np.float64),
            np.array(cim, np.float64), top)


def pauli_to_dia_host(terms, nq=None, *, big_endian=False):
    """H = sum_t c_t P_t (terms: [(coef, "X0 Y1 Z3"), ...] or QubitOperator
    text) on the host (dia_pauli_to_dia).  Qubit k is bit k of the basis
    index (big_endian=True: bit nq-1-k, OpenFermion's ordering).  Returns
    (n, offsets int32 [K], vals complex64 [K, stride], is_real)."""
    if isinstance(terms, str):
        terms = parse_pauli_sum(terms)
    if nq is None:
        nq = max(1, _pauli_masks(terms, None, False)[4])
    x, z, cre, cim, _ = _pauli_masks(terms, nq, big_endian)
    L = lib()
    pa = lambda a: a.ctypes.data_as(C.c_void_p)
    K = C.c_int(0)
    check(L.dia_pauli_to_dia(nq, len(terms), pa(x), pa(z), pa(cre), pa(cim), C.byref(K), None,
                             None, 0, None))
    n = 1 << nq
    stride = round_stride(n)
    offs = np.empty(max(K.value, 1), np.int32)
    vals = np.empty((max(K.value, 1), stride), np.complex64)
    real = C.c_int(0)
    check(L.dia_pauli_to_dia(nq, len(terms), pa(x), pa(z), pa(cre), pa(cim), C.byref(K),
                             pa(offs), pa(vals), stride, C.byref(real)))
    return n, offs[:K.value], vals[:K.value], bool(real.value)


def pauli_to_dia(terms, nq=None, *, big_endian=False, device="cuda", real="auto"):
    """The Hamiltonian as a whole-matrix DiaRows: float32 when it is real
    (real="auto") or real=True, else complex64 (for spmv_c64 /
    expm_taylor_c64)."""
    n, offs, vals, is_real = pauli_to_dia_host(terms, nq, big_endian=big_endian)
    as_real = is_real if real == "auto" else bool(real)
    if as_real and not is_real:
        raise DiaError(DIA_ERR_INVALID, "pauli_to_dia: the operator has imaginary entries")
    A = DiaRows.empty(n, n, offs, device=device,
                      dtype=torch.float32 if as_real else torch.complex64)
    if len(offs):
        A.vals.copy_(torch.from_numpy(vals.real.copy() if as_real else vals))
    return A


def read_mtx_host(path):
    """Parse a Matrix Market coordinate file into the rows layout on the host
    (dia_mtx_read; no GPU needed).  Returns (n_rows, n_cols, offsets int32
    [K], vals float32 [K, stride]) with stride = round_stride(n_rows)."""
    L = lib()
    bpath = os.fsencode(path)
    nr, nc, K = C.c_int64(0), C.c_int64(0), C.c_int(0)
    check(L.dia_mtx_read(bpath, C.byref(nr), C.byref(nc), C.byref(K), None, None, 0))
    offs = np.empty(max(K.value, 1), np.int32)
    stride = round_stride(nr.value)
    vals = np.empty((max(K.value, 1), stride), np.float32)
    check(L.dia_mtx_read(bpath, C.byref(nr), C.byref(nc), C.byref(K),
                         offs.ctypes.data_as(C.c_void_p), vals.ctypes.data_as(C.c_void_p),
                         stride))
    return nr.value, nc.value, offs[:K.value], vals[:K.value]


def read_mtx_c64_host(path):
    """Parse a Matrix Market coordinate file -- complex (general, symmetric,
    skew-symmetric, hermitian) or real -- into complex64 rows on the host
    (dia_mtx_read_c64).  Returns (n_rows, n_cols, offsets int32 [K], vals
    complex64 [K, stride], is_complex)."""
    L = lib()
    bpath = os.fsencode(path)
    nr, nc, K, cx = C.c_int64(0), C.c_int64(0), C.c_int(0), C.c_int(0)
    check(L.dia_mtx_read_c64(bpath, C.byref(nr), C.byref(nc), C.byref(K), None, None, 0,
                             C.byref(cx)))
    offs = np.empty(max(K.value, 1), np.int32)
    stride = round_stride(nr.value)
    vals = np.empty((max(K.value, 1), stride), np.complex64)
    check(L.dia_mtx_read_c64(bpath, C.byref(nr), C.byref(nc), C.byref(K),
                             offs.ctypes.data_as(C.c_void_p), vals.ctypes.data_as(C.c_void_p),
                             stride, C.byref(cx)))
    return nr.value, nc.value, offs[:K.value], vals[:K.value], bool(cx.value)


def write_mtx(path, n_rows, n_cols, offsets, vals):
    """Write a host rows-layout matrix (offsets [K], vals float32 [K, stride])
    as a Matrix Market coordinate file (dia_mtx_write)."""
    offsets = np.ascontiguousarray(offsets, np.int32)
    vals = np.ascontiguousarray(vals, np.float32)
    check(lib().dia_mtx_write(os.fsencode(path), n_rows, n_cols, len(offsets),
                              offsets.ctypes.data_as(C.c_void_p),
                              vals.ctypes.data_as(C.c_void_p), vals.shape[1] if vals.ndim == 2 else 0))


def read_mtx(path, *, device="cuda") -> DiaRows:
    """A Matrix Market coordinate file as a whole-matrix DiaRows on the GPU."""
    n_rows, n_cols, offs, vals = read_mtx_host(path)
    A = DiaRows.empty(n_rows, n_cols, offs, device=device)
    if len(offs):
        A.vals.copy_(torch.from_numpy(vals))
    return A


def read_mtx_c64(path, *, device="cuda") -> DiaRows:
    """A Matrix Market coordinate file as a complex64 whole-matrix DiaRows
    on the GPU (for spmv_c64 / expm_taylor_c64)."""
    n_rows, n_cols, offs, vals, _ = read_mtx_c64_host(path)
    A = DiaRows.empty(n_rows, n_cols, offs, device=device, dtype=torch.complex64)
    if len(offs):
        A.vals.copy_(torch.from_numpy(vals))
    return A


def expm_taylor(A: DiaRows, t, m, x, y=None, *, work=None, stream=None):
    """y = sum_{j=0}^{m} (tA)^j x / j!  (truncated Taylor series of exp(tA) x),
    one fused SpMV + scale + running-sum launch per term (dia_expm_taylor).
    A is a whole square matrix (vrow0 = 0); work (2n floats) may be passed
    to reuse scratch across calls, e.g. under CUDA graph capture."""
    if A.vrow0 != 0 or A.nrows != A.n_rows or A.n_rows != A.n_cols:
        raise DiaError(DIA_ERR_INVALID, "expm_taylor: A must be a whole square matrix")
    n = A.n_rows
    y = torch.empty(n, dtype=torch.float32, device=x.device) if y is None else y
    work = torch.empty(2 * n, dtype=torch.float32, device=x.device) if work is None else work
    with torch.cuda.device(x.device):
        check(lib().dia_expm_taylor(n, A.K, _dptr(A.d_offsets), _dptr(A.vals), A.stride,
                                    float(t), int(m), _dptr(x, torch.float32),
                                    _dptr(y, torch.float32), _dptr(work, torch.float32),
                                    _stream(stream)))
    return y


def spmspm_symbolic_device(n, d_A_off, d_nA, nA_cap, d_B_off, nC_cap, *, stream=None):
    """Output offsets of C = A*B computed on the device (dia_spmspm_symbolic_device).

    d_A_off (int32, capacity nA_cap) and d_nA (int32 [1]) are device
    tensors, d_B_off the device offsets of B.  Returns device tensors
    (C_off [nC_cap], nC [1]) without synchronising; nC[0] > nC_cap means the
    capacity was too small."""
    dev = d_A_off.device
    C_off = torch.zeros(max(nC_cap, 1), dtype=torch.int32, device=dev)
    nC = torch.zeros(1, dtype=torch.int32, device=dev)
    L = lib()
    ws = L.dia_spmspm_device_workspace(n, nA_cap, len(d_B_off), nC_cap)
    if ws < 0:
        raise DiaError(DIA_ERR_INVALID, "dia_spmspm_device_workspace: bad sizes")
    work = torch.empty(max(ws, 1), dtype=torch.uint8, device=dev)
    with torch.cuda.device(dev):
        check(L.dia_spmspm_symbolic_device(n, _dptr(d_A_off, torch.int32), _dptr(d_nA, torch.int32),
                                           nA_cap, _dptr(d_B_off, torch.int32), len(d_B_off),
                                           _dptr(C_off), _dptr(nC), nC_cap, _dptr(work), ws,
                                           _stream(stream)))
    return C_off, nC


class PowerChain:
    """Matrix-power chain P_{k+1} = P_k * H entirely on the device.

    H is a whole matrix (vrow0 = 0) with few diagonals.  Each step() runs
    dia_spmspm_rows_device: the output offsets (sumset) and the pair lists
    are built on the GPU, so no step synchronises with the host.  P_k lives
    in one of two ping-pong buffers of max_diags diagonals; power() returns
    the current P_k (it reads the diagonal count, one synchronisation, and
    the returned matrix shares the buffer the step after next overwrites).
    Results equal repeated spmspm(P, H) bit for bit."""

    def __init__(self, H: DiaRows, max_diags: int, *, stream=None):
        if H.vrow0 != 0 or H.nrows != H.n_rows or H.n_rows != H.n_cols:
            raise DiaError(DIA_ERR_INVALID, "PowerChain: H must be a whole square matrix")
        self.H, self.n, self.cap = H, H.n_rows, int(max_diags)
        if self.cap < H.K:
            raise DiaError(DIA_ERR_INVALID, "PowerChain: max_diags below H's diagonal count")
        dev = H.vals.device
        stride = round_stride(self.n)
        self._vals = [torch.zeros((self.cap, stride), dtype=torch.float32, device=dev)
                      for _ in range(2)]
        self._off = [torch.zeros(self.cap, dtype=torch.int32, device=dev) for _ in range(2)]
        self._cnt = [torch.zeros(1, dtype=torch.int32, device=dev) for _ in range(2)]
        self.reset()
        self._ws = lib().dia_spmspm_device_workspace(self.n, self.cap, H.K, self.cap)
        self._work = torch.empty(max(self._ws, 1), dtype=torch.uint8, device=dev)

    def reset(self):
        """Back to P_1 = H (device copies only)."""
        H = self.H
        w = min(self._vals[0].shape[1], H.stride)
        self._vals[0][:H.K, :w] = H.vals[:, :w]
        self._off[0][:H.K] = H.d_offsets
        self._cnt[0].fill_(H.K)
        self.k, self._cur = 1, 0

    def step(self, stream=None):
        a, b = self._cur, 1 - self._cur
        H = self.H
        with torch.cuda.device(H.vals.device):
            check(lib().dia_spmspm_rows_device(
                self.n, _dptr(self._off[a]), _dptr(self._cnt[a]), self.cap, _dptr(self._vals[a]),
                self._vals[a].shape[1], _dptr(H.d_offsets), H.K, _dptr(H.vals), H.stride,
                _dptr(self._off[b]), _dptr(self._cnt[b]), self.cap, _dptr(self._vals[b]),
                self._vals[b].shape[1], _dptr(self._work), self._ws, _stream(stream)))
        self._cur, self.k = b, self.k + 1

    def count(self):
        """Device tensor [1] holding the current power's diagonal count."""
        return self._cnt[self._cur]

    def power(self) -> DiaRows:
        nc = int(self._cnt[self._cur].item())
        if nc > self.cap:
            raise DiaError(DIA_ERR_CAPACITY, f"PowerChain: P_{self.k} has {nc} diagonals, "
                                             f"max_diags is {self.cap}")
        d_off = self._off[self._cur][:nc]
        return DiaRows(self.n, self.n, d_off.cpu().numpy().astype(np.int32), d_off,
                       self._vals[self._cur][:nc], 0, self.n)


class SpmspmPlan:
    """Reusable plan for C = A*B on the rows layout (dia_spmspm_plan_*).

    Fixes the offsets and buffer geometry of A (rows [A.vrow0, +A.nrows)),
    B (rows [b_lo, b_hi) of the block B) and C (same rows as A).  Creating it
    runs the symbolic phase and uploads the tables; execute() launches only
    kernels (the shared-memory-tiled kernel on the interior rows when the
    offsets allow it, the generic kernel elsewhere)."""

    def __init__(self, A: DiaRows, B: DiaRows, *, b_lo=None, b_hi=None):
        b_lo = B.vrow0 if b_lo is None else b_lo
        b_hi = B.vrow0 + B.nrows if b_hi is None else b_hi
        self._h = C.c_void_p()
        a_off = np.ascontiguousarray(A.offsets, np.int32)
        b_off = np.ascontiguousarray(B.offsets, np.int32)
        pa = lambda x: x.ctypes.data_as(C.c_void_p)
        with torch.cuda.device(A.vals.device):
            check(lib().dia_spmspm_plan_create(A.n_rows, pa(a_off), len(a_off), pa(b_off),
                                               len(b_off), A.stride, B.stride, A.stride,
                                               A.vrow0, A.nrows, B.vrow0, b_lo, b_hi,
                                               C.byref(self._h)))
        nc = C.c_int(0)
        check(lib().dia_spmspm_plan_info(self._h, C.byref(nc), None, None, None, None, None,
                                         None))
        self.C_off = np.empty(nc.value, np.int32)
        tr, tlo, thi = C.c_int(0), C.c_int64(0), C.c_int64(0)
        check(lib().dia_spmspm_plan_info(self._h, None, pa(self.C_off), None, None,
                                         C.byref(tr), C.byref(tlo), C.byref(thi)))
        self.tile_rows, self.tiled = tr.value, (tlo.value, thi.value)
        self.A, self.B = A, B

    def new_C(self, zero=True):
        A = self.A
        return DiaRows.empty(A.n_rows, A.n_cols, self.C_off, vrow0=A.vrow0, nrows=A.nrows,
                             device=A.vals.device, zero=zero)

    def execute(self, A, B, C_out, row_lo=None, row_hi=None, *, use_tiles=True, stream=None):
        lo = A.vrow0 if row_lo is None else row_lo
        hi = A.vrow0 + A.nrows if row_hi is None else row_hi
        check(lib().dia_spmspm_plan_execute(self._h, _dptr(A.vals), _dptr(B.vals),
                                            _dptr(C_out.vals), lo, hi, int(use_tiles),
                                            _stream(stream)))
        return C_out

    def __del__(self):
        if getattr(self, "_h", None) and self._h.value and _lib is not None:
            _lib.dia_spmspm_plan_destroy(self._h)
            self._h = C.c_void_p()


def spmspm(A: DiaRows, B: DiaRows, C_out: DiaRows | None = None, *, b_lo=None, b_hi=None,
           symbolic=None, method="auto", stream=None):
    """C = A*B on the rows layout.  A and C cover the same row block; B may
    be a wider block (the halo rows of a partitioned product).
    method: "auto"/"tiled" plan the product (tiled kernel where possible),
    "planned_generic" plans it but keeps the generic kernel, "generic" runs
    the unplanned entry point (device-side pair resolution)."""
    n = A.n_rows
    if method != "generic":
        plan = SpmspmPlan(A, B, b_lo=b_lo, b_hi=b_hi)
        if C_out is None:
            C_out = plan.new_C()
        return plan.execute(A, B, C_out, use_tiles=method != "planned_generic", stream=stream)
    if symbolic is None:
        symbolic = spmspm_symbolic(n, A.offsets, B.offsets)
    if C_out is None:
        C_out = DiaRows.empty(n, n, symbolic["C_off"], vrow0=A.vrow0, nrows=A.nrows,
                              device=A.vals.device, zero=True)
    b_lo = B.vrow0 if b_lo is None else b_lo
    b_hi = B.vrow0 + B.nrows if b_hi is None else b_hi
    check(lib().dia_spmspm_rows(n, _dptr(A.vals), A.stride, _dptr(A.d_offsets), A.K,
                                _dptr(B.vals), B.stride, B.vrow0, b_lo, b_hi,
                                _dptr(B.d_offsets), B.K, _dptr(C_out.vals), C_out.stride,
                                _dptr(C_out.d_offsets), C_out.K, A.vrow0, A.vrow0,
                                A.vrow0 + A.nrows, _stream(stream)))
    return C_out


# ---------------------------------------------------------------- gemm_diag

def gemm_diag(DA, DB, off_A, off_B, n, C_data, C_offsets, C_lens, k_to_idx, *, beta=1,
              mode=GEMM_AUTO, h_off_A=None, h_off_B=None, stream=None):
    """gemm_diag product on the reference's layouts (device tensors).
    beta=1 accumulates into C_data like the reference; beta=0 overwrites."""
    hA = None if h_off_A is None else np.ascontiguousarray(h_off_A, np.int32)
    hB = None if h_off_B is None else np.ascontiguousarray(h_off_B, np.int32)
    check(lib().dia_gemm_diag_ex(_dptr(DA, torch.float32), _dptr(DB, torch.float32),
                                 _dptr(off_A, torch.int32), _dptr(off_B, torch.int32),
                                 None if hA is None else hA.ctypes.data_as(C.c_void_p),
                                 None if hB is None else hB.ctypes.data_as(C.c_void_p),
                                 off_A.numel(), off_B.numel(), n, _dptr(C_data, torch.float32),
                                 _dptr(C_offsets, torch.int32), _dptr(C_lens, torch.int32),
                                 _dptr(k_to_idx, torch.int32), beta, mode, _stream(stream)))
    return C_data


def gemm_diag_layout(n, off_A, off_B):
    """C layout of gemm_diag (build_c_layout, gemm_diag/gemm_diag.cu:387-423):
    int value starts, lengths, k_to_idx[2n-1], ascending k list, total."""
    sym = spmspm_symbolic(n, off_A, off_B)
    k_list = sym["C_off"]
    starts = sym["C_start"]
    if len(starts) and int(starts[-1]) + int(sym["C_len"][-1]) >= 2 ** 31:
        raise DiaError(DIA_ERR_UNSUPPORTED, "gemm_diag layout uses int value starts")
    k2i = np.full(2 * n - 1, -1, np.int32)
    k2i[k_list + n - 1] = np.arange(len(k_list), dtype=np.int32)
    total = int(sym["C_len"].astype(np.int64).sum())
    return starts.astype(np.int32), sym["C_len"], k2i, k_list, total


def device_status(clear=True):
    """Status bits set by kernels that gave up a bounded wait (0 = none)."""
    v = C.c_uint(0)
    check(lib().dia_device_status(C.byref(v), int(clear)))
    return v.value
