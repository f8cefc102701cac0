"""gemm_diag parity on the GPU (reference argument set, C ABI).

SIMT mode is exact fp32 in cpu_diag_multiply's order; the tensor-core mode
computes in TF32 and is held to relative L2 <= 5e-3 against an fp64
accumulation (the tolerance the north star states for TF32)."""
import numpy as np
import pytest
import torch

import diagpu_b200 as dg
import oracle
from tests._util import dev, rel_l2, same

pytestmark = pytest.mark.gpu

TF32_TOL = 5e-3


def _run(DA, DB, off, n, layout, mode, beta=1, C0=None):
    co, cl, k2i, kl, tot = layout
    C = torch.zeros(tot, device="cuda") if C0 is None else dev(C0)
    dg.gemm_diag(dev(DA), dev(DB), dev(off), dev(off), n, C, dev(co), dev(cl), dev(k2i),
                 beta=beta, mode=mode)
    return C.cpu().numpy()


def test_golden_simt(golden):
    g = golden["gemm_diag"]
    for name in g["names"]:
        off = g[f"{name}__off"]
        n = g[f"{name}__DA"].size // len(off)
        layout = oracle.build_c_layout(n, off, off)
        got = _run(g[f"{name}__DA"], g[f"{name}__DB"], off, n, layout, dg.GEMM_SIMT)
        assert same(got, g[f"{name}__C"]), name


def test_beta_semantics():
    rng = np.random.default_rng(3)
    n, off = 999, np.arange(-5, 6, dtype=np.int32)
    DA = rng.uniform(-1, 1, (len(off), n)).astype(np.float32)
    DB = rng.uniform(-1, 1, (len(off), n)).astype(np.float32)
    layout = oracle.build_c_layout(n, off, off)
    C0 = rng.uniform(-1, 1, layout[4]).astype(np.float32)
    acc = _run(DA, DB, off, n, layout, dg.GEMM_SIMT, beta=1, C0=C0)
    ovw = _run(DA, DB, off, n, layout, dg.GEMM_SIMT, beta=0, C0=C0)
    ref = oracle.gemm_diag(DA, off, DB, off, n, f64=False)[0]
    assert same(ovw, ref)
    assert same(acc, (C0 + ovw).astype(np.float32))


def test_noncontiguous_offsets_simt():
    rng = np.random.default_rng(4)
    n = 3001
    offA = np.array([-700, -3, 0, 2, 45], np.int32)
    offB = np.array([9, -1, 0, 800], np.int32)
    DA = rng.uniform(-1, 1, (len(offA), n)).astype(np.float32)
    DB = rng.uniform(-1, 1, (len(offB), n)).astype(np.float32)
    co, cl, k2i, kl, tot = oracle.build_c_layout(n, offA, offB)
    C = torch.zeros(tot, device="cuda")
    dg.gemm_diag(dev(DA), dev(DB), dev(offA), dev(offB), n, C, dev(co), dev(cl), dev(k2i),
                 mode=dg.GEMM_SIMT)
    ref = np.zeros(tot, np.float32)
    import oracle as O
    O.lib().orc_gemm_diag_f32(DA.reshape(-1), offA, len(offA), DB.reshape(-1), offB, len(offB),
                              n, ref, co, k2i)
    assert same(C.cpu().numpy(), ref)


def _config4(n=262144, hb=64):
    off = np.arange(-hb, hb + 1, dtype=np.int32)
    A = dg.DiaRows.synth(n, n, off, seed=401)
    B = dg.DiaRows.synth(n, n, off, seed=402)
    # row-packed DA[ri*n + row]: the rows layout with stride n
    DA = A.vals[:, :n].contiguous()
    DB = B.vals[:, :n].contiguous()
    return off, DA, DB


@pytest.mark.parametrize("mode", [dg.GEMM_SIMT, dg.GEMM_AUTO])
def test_config4_dense_band(mode):
    """Config 4: n = 262144, offsets -64..64, C 257 diagonals."""
    n = 262144
    off, DA, DB = _config4(n)
    co, cl, k2i, kl, tot = oracle.build_c_layout(n, off, off)
    C = torch.zeros(tot, device="cuda")
    dg.gemm_diag(DA, DB, dev(off), dev(off), n, C, dev(co), dev(cl), dev(k2i), mode=mode)
    got = C.cpu().numpy()
    ref64, _ = oracle.gemm_diag(DA.cpu().numpy(), off, DB.cpu().numpy(), off, n, f64=True)
    err = rel_l2(got, ref64)
    assert err <= (1e-6 if mode == dg.GEMM_SIMT else TF32_TOL), err


@pytest.mark.parametrize("n,lo_a,P,lo_b,Q", [(256, -4, 9, -4, 9), (1000, -64, 129, -64, 129),
                                            (777, -3, 5, 2, 40), (130, 0, 1, 0, 1),
                                            (5000, -20, 41, -100, 120),
                                            (2048, -20, 40, -15, 30),
                                            (3000, -10, 60, -70, 145)])
def test_tcgen05_small_bands(n, lo_a, P, lo_b, Q):
    """Tensor-core mode on contiguous bands: ragged last tile, asymmetric
    and one-diagonal bands, the widest supported B band, tiles whose
    accumulator splits into two unequal or B-limited column halves."""
    offA = np.arange(lo_a, lo_a + P, dtype=np.int32)
    offB = np.arange(lo_b, lo_b + Q, dtype=np.int32)
    DA = dg.DiaRows.synth(n, n, offA, seed=11).vals[:, :n].contiguous()
    DB = dg.DiaRows.synth(n, n, offB, seed=12).vals[:, :n].contiguous()
    co, cl, k2i, kl, tot = oracle.build_c_layout(n, offA, offB)
    for beta in (0, 1):
        C0 = torch.full((tot,), 0.5, device="cuda")
        dg.gemm_diag(DA, DB, dev(offA), dev(offB), n, C0, dev(co), dev(cl), dev(k2i),
                     mode=dg.GEMM_TCGEN05, beta=beta)
        torch.cuda.synchronize()
        assert dg.device_status() == 0
        ref = np.zeros(tot, np.float64)
        oracle.lib().orc_gemm_diag_f64(DA.cpu().numpy().reshape(-1), offA, P,
                                       DB.cpu().numpy().reshape(-1), offB, Q, n, ref, co, k2i,
                                       oracle.threads())
        got = C0.cpu().numpy().astype(np.float64) - (0.5 if beta else 0.0)
        assert rel_l2(got, ref) <= TF32_TOL, (beta, rel_l2(got, ref))


def test_tcgen05_rejects_wide_bands_auto_falls_back():
    n = 2000
    off = np.arange(-150, 151, dtype=np.int32)          # P + Q - 1 = 601 > 257
    DA = dg.DiaRows.synth(n, n, off, seed=1).vals[:, :n].contiguous()
    co, cl, k2i, kl, tot = oracle.build_c_layout(n, off, off)
    C = torch.zeros(tot, device="cuda")
    with pytest.raises(dg.DiaError) as e:
        dg.gemm_diag(DA, DA, dev(off), dev(off), n, C, dev(co), dev(cl), dev(k2i),
                     mode=dg.GEMM_TCGEN05)
    assert e.value.code == dg.DIA_ERR_UNSUPPORTED
    dg.gemm_diag(DA, DA, dev(off), dev(off), n, C, dev(co), dev(cl), dev(k2i), beta=0)
    ref = oracle.gemm_diag(DA.cpu().numpy(), off, DA.cpu().numpy(), off, n, f64=False)[0]
    assert same(C.cpu().numpy(), ref)   # AUTO took the exact SIMT path


def test_tcgen05_wait_runs_out_and_the_gpu_stays_usable():
    """Failure detection without a fault: with a 1 ms wait limit and one
    operand-ready arrival withheld, the tcgen05 kernel's MMA issuer gives up,
    every role stops, issued copies drain, tensor memory is freed and
    DIA_TC_TIMEOUT is reported.  The next normal call is correct."""
    n = 4096
    off = np.arange(-4, 5, dtype=np.int32)
    DA = dg.DiaRows.synth(n, n, off, seed=21).vals[:, :n].contiguous()
    DB = dg.DiaRows.synth(n, n, off, seed=22).vals[:, :n].contiguous()
    co, cl, k2i, kl, tot = oracle.build_c_layout(n, off, off)
    L = dg.lib()
    dg.device_status(clear=True)
    C = torch.zeros(tot, device="cuda")
    dg.check(L.dia_test_tc_wait(1_000_000, 1))
    try:
        dg.gemm_diag(DA, DB, dev(off), dev(off), n, C, dev(co), dev(cl), dev(k2i),
                     mode=dg.GEMM_TCGEN05, beta=0)
        torch.cuda.synchronize()
    finally:
        dg.check(L.dia_test_tc_wait(0, 0))
    assert dg.device_status(clear=True) & dg.DIA_TC_TIMEOUT
    C.zero_()
    dg.gemm_diag(DA, DB, dev(off), dev(off), n, C, dev(co), dev(cl), dev(k2i),
                 mode=dg.GEMM_TCGEN05, beta=0)
    torch.cuda.synchronize()
    assert dg.device_status() == 0
    ref = oracle.gemm_diag(DA.cpu().numpy(), off, DB.cpu().numpy(), off, n, f64=True)[0]
    assert rel_l2(C.cpu().numpy(), ref) <= TF32_TOL
