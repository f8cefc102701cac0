"""dia_spmspm_hm_noalloc: the SpMSpM entry point for callers that cannot
allocate device memory while they run (for example an application whose
allocator has already reserved all device memory).  It keeps its pair plan in
a fixed library-owned device array instead of allocating scratch, so it is
checked here against dia_spmspm_hm, the allocating entry point, through the
C ABI: two different products back to back (the second must not be affected
by what the first left in the shared array), results equal bit for bit (the
tolerance of the other FP32 tests), plus the size limit.

This file is collected last on purpose (test_zz_*)."""
import ctypes as C

import numpy as np
import pytest
import torch

import diagpu_b200 as dg
from tests._util import dev, same

pytestmark = pytest.mark.gpu


def _hm(g, name, tag):
    return tuple(g[f"{name}__{tag}_{f}"] for f in ("off", "len", "start", "val"))


def _args(n, A, B, Cs, Cv):
    lk = np.full(2 * n - 1, -1, np.int32)
    for i, d in enumerate(B[0]):
        lk[d + n - 1] = i
    keep = [dev(A[3]), dev(A[2]), dev(A[0]), dev(A[1]), dev(B[3]), dev(B[2]), dev(B[1]),
            dev(lk), dev(Cs[2]), dev(Cs[0]), dev(Cs[1])]
    p = lambda t: C.c_void_p(t.data_ptr())
    a = [p(keep[0]), p(keep[1]), p(keep[2]), p(keep[3]), len(A[0]), p(keep[4]), p(keep[5]),
         p(keep[6]), p(keep[7]), p(Cv), p(keep[8]), p(keep[9]), p(keep[10]), len(Cs[0]), n,
         C.c_void_p(torch.cuda.current_stream().cuda_stream)]
    return a, keep


def _run(fn, n, A, B, Cs):
    nnz = int(Cs[2][-1] + Cs[1][-1])
    Cv = torch.full((nnz,), np.nan, device="cuda")
    a, keep = _args(n, A, B, Cs, Cv)
    dg.check(fn(*a))
    torch.cuda.synchronize()
    return Cv.cpu().numpy()


def test_noalloc_matches_allocating_entry_point_twice(golden):
    L = dg.lib()
    cases = [(golden["spmspm_scatter"], "n600_k32"), (golden["spmspm_banded"], "n1000_w16")]
    for g, name in cases:
        A, B = _hm(g, name, "A"), _hm(g, name, "B")
        n = int(A[1][A[0] == 0][0])
        Cs = (g[f"{name}__C_off"], g[f"{name}__C_len"], g[f"{name}__C_start"])
        ref = _run(L.dia_spmspm_hm, n, A, B, Cs)
        got = _run(L.dia_spmspm_hm_noalloc, n, A, B, Cs)
        assert same(got, ref), name
        assert same(got, g[f"{name}__C_val"]), name


def test_noalloc_rejects_plans_beyond_the_static_buffer():
    L = dg.lib()
    n = 4096
    offs = np.arange(-2047, 2048, dtype=np.int32)          # 4095 diagonals
    ln = (n - np.abs(offs)).astype(np.int32)
    st = np.concatenate([[0], np.cumsum(ln[:-1], dtype=np.int64)]).astype(np.int64)
    A = (offs, ln, st, np.zeros(int(ln.sum()), np.float32))
    Cs = (offs, ln, st)                                    # 4095 x 4095 x 24 B > 8 MiB
    Cv = torch.zeros(int(ln.sum()), device="cuda")
    a, keep = _args(n, A, A, Cs, Cv)
    rc = L.dia_spmspm_hm_noalloc(*a)
    assert rc == dg.DIA_ERR_CAPACITY
    assert "static buffer" in L.dia_last_error().decode()


def _device_memory_state():
    """(free bytes, mempool reserved bytes, mempool used bytes) of the current
    device, read through the driver API: cuMemGetInfo and the attributes of
    the device's current memory pool, the pool cudaMallocAsync draws from."""
    cu = C.CDLL("libcuda.so.1")
    free, total = C.c_size_t(0), C.c_size_t(0)
    assert cu.cuMemGetInfo_v2(C.byref(free), C.byref(total)) == 0
    dev, pool = C.c_int(0), C.c_void_p()
    assert cu.cuCtxGetDevice(C.byref(dev)) == 0
    assert cu.cuDeviceGetMemPool(C.byref(pool), dev) == 0
    reserved, used = C.c_uint64(0), C.c_uint64(0)
    assert cu.cuMemPoolGetAttribute(pool, 5, C.byref(reserved)) == 0   # RESERVED_MEM_CURRENT
    assert cu.cuMemPoolGetAttribute(pool, 7, C.byref(used)) == 0       # USED_MEM_CURRENT
    return free.value, reserved.value, used.value


def test_noalloc_leaves_device_memory_untouched(golden):
    """The property the entry point exists for: a call changes neither the
    device's free memory nor the stream-ordered pool, while the allocating
    entry point draws its scratch from that pool."""
    L = dg.lib()
    g, name = golden["spmspm_scatter"], "n600_k32"
    A, B = _hm(g, name, "A"), _hm(g, name, "B")
    n = int(A[1][A[0] == 0][0])
    Cs = (g[f"{name}__C_off"], g[f"{name}__C_len"], g[f"{name}__C_start"])
    nnz = int(Cs[2][-1] + Cs[1][-1])
    Cv = torch.zeros(nnz, device="cuda")
    a, keep = _args(n, A, B, Cs, Cv)
    dg.check(L.dia_spmspm_hm_noalloc(*a))     # first call on the device: address lookup
    torch.cuda.synchronize()
    before = _device_memory_state()
    for _ in range(3):
        dg.check(L.dia_spmspm_hm_noalloc(*a))
    torch.cuda.synchronize()
    assert _device_memory_state() == before
    dg.check(L.dia_spmspm_hm(*a))
    torch.cuda.synchronize()
    used_high = C.c_uint64(0)
    cu = C.CDLL("libcuda.so.1")
    dev, pool = C.c_int(0), C.c_void_p()
    cu.cuCtxGetDevice(C.byref(dev))
    cu.cuDeviceGetMemPool(C.byref(pool), dev)
    assert cu.cuMemPoolGetAttribute(pool, 8, C.byref(used_high)) == 0   # USED_MEM_HIGH
    assert used_high.value > 0, "the allocating entry point should draw from the pool"
