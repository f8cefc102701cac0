"""DIA SpMV / SpMSpM benchmark on B200 (one process per GPU).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Headline (the JSON line's `value`): FP32 DIA SpMV y = A*x on config 5 (3D
27-point stencil, 256x256x1024, n = 67,108,864, 27 diagonals), A
row-partitioned over N GPUs with a +-65,793-column x halo exchanged over
NCCL (strong scaling: the matrix is fixed, each GPU gets n/N rows).
`value` = algorithmic bytes 4*(nnz + 2n) of the whole matrix / max-over-ranks
step time, in GB/s.  `secondary` holds C = A*A on the same matrix (useful
GFLOP/s and byte roofline) and, at N = 1, configs 1-4.

Inputs are generated on the device by the library's counter-based generator
(seeded, uniform [-1, 1]); every timed input is larger than the 126 MB L2
except config 1, which is timed per launch with an L2 flush in between.

--impl reference times the reference's own CPU SpMV (spmv_from_recon,
spmv/test/test_tc_spmv.cu:64-79, compiled from the reference sources into
oracle/_ref/) on the host cores, on a bounded row sample of config 5.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np
import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

N5 = 256 * 256 * 1024
OFF5 = np.array([i + 256 * j + 65536 * k for k in (-1, 0, 1) for j in (-1, 0, 1)
                 for i in (-1, 0, 1)], np.int32)
OFF2 = np.array([-16384, -128, -1, 0, 1, 128, 16384], np.int32)
SEED_A, SEED_X = 5001, 5002
REF_SAMPLE_ROWS = 4 * 1024 * 1024
# DRAM bytes (read + write) of one spmv_kernel launch on config 5, derived
# rather than measured by this run: the ncu capture of the 4,194,304-row case
# (471.4 MB) scaled by the ratio of algorithmic bytes (16.15)
SPMV5_TRAFFIC = 7_611_000_000


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def spmv_bytes(n, offsets, r0, r1):
    nnz = sum(max(0, min(r1, n - int(d)) - max(r0, -int(d))) for d in offsets)
    return 4 * (nnz + 2 * (r1 - r0)), nnz


# ------------------------------------------------------------------ clocks

class Clocks:
    """nvidia-smi sampling during the timed region."""

    def __init__(self, gpus):
        self.gpus = gpus
        self.proc = None
        self.path = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={q}", "--format=csv,noheader,nounits", "-lms",
                 "100"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        if self.proc is None or not self.path:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9 or not f[0].isdigit() or int(f[0]) not in self.gpus:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for nm, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        os.unlink(self.path)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "samples": len(sm),
                "reasons": sorted(reasons)}


# ---------------------------------------------------------------- timing

def timed(fn, steps, warmup, *, flush=None, per_launch=False, world=1):
    """Mean ms of fn() over `steps` after `warmup`, CUDA events on the
    current stream; with per_launch each call is bracketed by its own events
    and preceded by flush() and a ~50 us device sleep (both outside the
    bracket; the sleep keeps the GPU busy while the host enqueues the
    bracket, so the host's launch latency does not land inside it).  With world > 1 a barrier
    precedes the timed region, so a step that exchanges halos does not start
    its clock while the peer rank is still setting up."""
    for _ in range(warmup):
        fn()
    barrier(world)
    if per_launch:
        tot = 0.0
        for _ in range(steps):
            if flush is not None:
                flush()
            # keep the GPU busy while the host enqueues the bracket, so the
            # bracket holds device time only, not the host's launch latency
            torch.cuda._sleep(100_000)
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            fn()
            e.record()
            e.synchronize()
            tot += s.elapsed_time(e)
        return tot / steps
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(steps):
        fn()
    e.record()
    e.synchronize()
    return s.elapsed_time(e) / steps


def max_over_ranks(v, world):
    if world == 1:
        return v
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world):
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()


# ------------------------------------------------------------ workloads

def spmspm_useful(n, A_off, B_off, sym, r0, r1):
    """Exact useful flops 2 * sum over pairs of the rows in [r0, r1) where
    A[i, i+da], B[i+da, i+dc] and C[i, i+dc] all exist."""
    tot = 0
    for c, dc in enumerate(sym["C_off"]):
        for q in range(sym["pair_ptr"][c], sym["pair_ptr"][c + 1]):
            da = int(A_off[sym["pair_a"][q]])
            lo = max(r0, 0, -da, -int(dc))
            hi = min(r1, n, n - da, n - int(dc))
            tot += max(0, hi - lo)
    return 2 * tot


def nnz_rows(n, offs, r0, r1):
    return sum(max(0, min(r1, n - int(d)) - max(r0, -int(d))) for d in offs)


def tf32_peak_tflops(size=8192, reps=5):
    """Dense TF32 throughput of this GPU (cuBLAS fp32 GEMM, TF32 allowed):
    the denominator of gemm_diag's tensor-pipe fraction."""
    a = torch.randn(size, size, device="cuda")
    b = torch.randn(size, size, device="cuda")
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = True
    try:
        ms = timed(lambda: a @ b, reps, 2)
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    return 2 * size ** 3 / ms / 1e9


def l2_flusher():
    """Write a buffer larger than L2, then read another one: the write
    evicts the timed kernel's data, and the read pass evicts the dirty lines
    the write left, so their write-back happens here, outside the timed
    bracket, instead of inside the next timed launch."""
    wbuf = torch.empty(64 * 1024 * 1024, dtype=torch.float32, device="cuda")  # 256 MB > L2
    rbuf = torch.zeros(64 * 1024 * 1024, dtype=torch.float32, device="cuda")

    def flush():
        wbuf.zero_()
        rbuf.sum()
    return flush


def roofline(achieved_gbs, hbm, src, traffic=None):
    return {"bound": "hbm", "achieved": round(achieved_gbs, 1), "peak": hbm, "unit": "GB/s",
            "frac": round(achieved_gbs / hbm, 4), "peak_source": src, "traffic": traffic}


def hm_of(A):
    """The HM arrays (values, int64 starts, offsets, lengths) of a whole
    rows-layout matrix, on the device."""
    n = A.n_rows
    ln = (n - np.abs(A.offsets.astype(np.int64))).astype(np.int64)
    st = np.concatenate([[0], np.cumsum(ln[:-1])]).astype(np.int64)
    val = torch.empty(int(ln.sum()), device="cuda")
    for k, d in enumerate(A.offsets):
        r0 = -min(int(d), 0)
        val[int(st[k]):int(st[k] + ln[k])] = A.vals[k, r0:r0 + int(ln[k])]
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    return val, t(st), t(A.offsets.astype(np.int32)), t(ln.astype(np.int32))


def secondary_spmspm(dg, name, n, A, B, steps, warmup, hbm, src, flush=None):
    sym = dg.spmspm_symbolic(n, A.offsets, B.offsets)
    plan = dg.SpmspmPlan(A, B)
    Cm = plan.new_C()
    fn = lambda: plan.execute(A, B, Cm)
    ms = timed(fn, steps, warmup, flush=flush, per_launch=flush is not None)
    # the same product through the reference's HM argument set (the
    # counterpart of gather_meta_kernel's launch)
    av, ast, aoff, aln = hm_of(A)
    bv, bst, boff, bln = (av, ast, aoff, aln) if B is A else hm_of(B)
    lk = np.full(2 * n - 1, -1, np.int32)
    lk[B.offsets.astype(np.int64) + n - 1] = np.arange(B.K, dtype=np.int32)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    dlk, dcs = t(lk), t(sym["C_start"].astype(np.int64))
    dco, dcl = t(sym["C_off"].astype(np.int32)), t(sym["C_len"].astype(np.int32))
    Chm = torch.empty(int(sym["C_len"].astype(np.int64).sum()), device="cuda")
    hm_ms = timed(lambda: dg.spmspm_hm(av, ast, aoff, aln, bv, bst, bln, dlk, Chm, dcs, dco, dcl,
                                       n), steps, warmup, flush=flush,
                  per_launch=flush is not None)
    del av, bv, Chm
    nnzA = nnz_rows(n, A.offsets, 0, n)
    nnzB = 0 if B is A else nnz_rows(n, B.offsets, 0, n)
    nnzC = int(sym["C_len"].astype(np.int64).sum())
    byts = 4 * (nnzA + nnzB + nnzC)
    fl = spmspm_useful(n, A.offsets, B.offsets, sym, 0, n)
    del Cm
    return {"workload": name, "metric": "spmspm_useful_GFLOPs", "value": round(fl / ms / 1e6, 2),
            "unit": "GFLOP/s", "ms": round(ms, 4), "bytes": byts, "useful_flops": fl,
            "c_diagonals": len(sym["C_off"]), "pairs": len(sym["pair_a"]),
            "hm_args_ms": round(hm_ms, 4),
            "roofline": roofline(byts / ms / 1e6, hbm, src), "gpu_launches_per_step": 2}


def single_gpu_extras(dg, steps, warmup, hbm, src):
    out = []
    flush = l2_flusher()
    # config 1: 2D Poisson SpMV (29 MB: L2-resident, flushed per launch)
    n = 1 << 20
    offs = np.array([-1024, -1, 0, 1, 1024], np.int32)
    A = dg.DiaRows.synth(n, n, offs, seed=101, base=[-1, -1, 4, -1, -1], lo=-0.01, hi=0.01)
    x = dg.synth_vector(n, seed=102)
    y = torch.empty(A.stride, device="cuda")
    ms = timed(lambda: dg.spmv(A, x, y), steps, warmup, flush=flush, per_launch=True)
    b, nnz = spmv_bytes(n, offs, 0, n)
    out.append({"workload": "config1 2D 5-pt Poisson n=1048576 SpMV (L2 flushed per launch)",
                "metric": "spmv_GBps", "value": round(b / ms / 1e6, 1), "unit": "GB/s",
                "ms": round(ms, 4), "bytes": b, "roofline": roofline(b / ms / 1e6, hbm, src),
                "gpu_launches_per_step": 1})
    del A, x, y
    # config 2: 3D 7-point stencil C = A*A
    n = 128 ** 3
    offs = np.array([-16384, -128, -1, 0, 1, 128, 16384], np.int32)
    A = dg.DiaRows.synth(n, n, offs, seed=201)
    out.append(secondary_spmspm(dg, "config2 3D 7-pt 128^3 C=A*A", n, A, A, steps, warmup, hbm,
                                src, flush=flush))
    del A
    # config 3: scattered 32 + 32 offsets, normal values
    n = 1_000_000
    rng = np.random.default_rng(301)

    def scat():
        s = {0}
        while len(s) < 32:
            s.add(int(rng.integers(-512, 513)))
        return np.array(sorted(s), np.int32)
    A = dg.DiaRows.synth(n, n, scat(), seed=303, kind=1, lo=0.0, hi=1.0)
    B = dg.DiaRows.synth(n, n, scat(), seed=304, kind=1, lo=0.0, hi=1.0)
    out.append(secondary_spmspm(dg, "config3 scattered 32x32 offsets n=1e6 C=A*B", n, A, B,
                                steps, warmup, hbm, src))
    del A, B
    # config 4: dense band gemm_diag (reference argument set)
    n, hb = 262144, 64
    goff = np.arange(-hb, hb + 1, dtype=np.int32)
    DA = dg.DiaRows.synth(n, n, goff, seed=401).vals[:, :n].contiguous()
    DB = dg.DiaRows.synth(n, n, goff, seed=402).vals[:, :n].contiguous()
    co, cl, k2i, kl, tot = dg.gemm_diag_layout(n, goff, goff)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    dco, dcl, dk2i, doff = t(co), t(cl), t(k2i), t(goff)
    C = torch.zeros(tot, device="cuda")
    fn = lambda: dg.gemm_diag(DA, DB, doff, doff, n, C, dco, dcl, dk2i, beta=0, h_off_A=goff,
                              h_off_B=goff)
    ms = timed(fn, max(3, steps // 4), warmup)
    byts = 4 * (2 * nnz_rows(n, goff, 0, n) + tot)
    sym = dg.spmspm_symbolic(n, goff, goff)
    fl = spmspm_useful(n, goff, goff, sym, 0, n)
    # TF32 peak of this GPU, measured: cuBLAS fp32 GEMM with TF32 tensor cores
    tf32 = tf32_peak_tflops()
    issued = 2 * 128 * 160 * 32 * ((n + 127) // 128) * 8   # 128x160x32 per chunk, 8 chunks a tile
    out.append({"workload": "config4 dense band hb=64 n=262144 gemm_diag (beta=0)",
                "metric": "gemm_diag_useful_GFLOPs", "value": round(fl / ms / 1e6, 2),
                "unit": "GFLOP/s", "ms": round(ms, 4), "bytes": byts, "useful_flops": fl,
                "roofline": roofline(byts / ms / 1e6, hbm, src), "mode": "auto",
                "tensor": {"tf32_peak_tflops_measured": round(tf32, 1),
                           "useful_tflops": round(fl / ms / 1e9, 2),
                           "issued_tflops": round(issued / ms / 1e9, 2),
                           "frac_useful": round(fl / ms / 1e9 / tf32, 4),
                           "frac_issued": round(issued / ms / 1e9 / tf32, 4),
                           "note": "16 useful flop per algorithmic byte: HBM-bound far below "
                                   "the TF32 ridge"}})
    del DA, DB, C
    # matrix-power chain H^8 of the config-1 operator, symbolic phase on the device
    fn, byts = _only_chain(dg)
    ms = timed(fn, max(3, steps // 10), min(warmup, 3))
    fnh, _ = _only_chain(dg, host=True)
    ms_host = timed(fnh, 3, 1)
    out.append({"workload": f"config1 operator power chain H^{CHAIN_K} ({CHAIN_K - 1} products, "
                            "device-side symbolic phase, no host synchronisation)",
                "metric": "chain_GBps", "value": round(byts / ms / 1e6, 1), "unit": "GB/s",
                "ms": round(ms, 4), "bytes": byts,
                "roofline": roofline(byts / ms / 1e6, hbm, src),
                "host_planned_ms": round(ms_host, 4)})
    # truncated-Taylor exp(tA) x of the config-1 operator: 16 chained SpMV terms
    fn, byts = _only_taylor(dg)
    ms = timed(fn, max(3, steps // 5), min(warmup, 3), flush=flush, per_launch=True)
    out.append({"workload": f"config1 operator exp(tA)x, truncated Taylor, {TAYLOR_M} fused "
                            "SpMV+scale+sum terms (L2 flushed per call)",
                "metric": "taylor_GBps", "value": round(byts / ms / 1e6, 1), "unit": "GB/s",
                "ms": round(ms, 4), "bytes": byts,
                "roofline": roofline(byts / ms / 1e6, hbm, src),
                "gpu_launches_per_step": TAYLOR_M})
    # Lanczos (eigenvalues of the symmetric config-1 operator), all on the device
    fn, byts = _only_lanczos(dg)
    ms = timed(fn, max(3, steps // 10), min(warmup, 3))
    out.append({"workload": f"config1 operator Lanczos, {LANCZOS_M} steps on the device "
                            "(fused SpMV+dot, fp64 fixed-order reductions, no host sync)",
                "metric": "lanczos_GBps", "value": round(byts / ms / 1e6, 1), "unit": "GB/s",
                "ms": round(ms, 4), "bytes": byts, "roofline": roofline(byts / ms / 1e6, hbm, src),
                "gpu_launches_per_step": 2 + 2 * LANCZOS_M})
    # complex64 SpMV (Hamiltonian-type operators), 27-point stencil on 256^3
    fn, byts = _only_spmv_c64(dg)
    ms = timed(fn, max(3, steps // 5), min(warmup, 3))
    out.append({"workload": "complex64 DIA SpMV, 27-pt stencil 256^3 (n=16.8M, inputs > L2)",
                "metric": "spmv_c64_GBps", "value": round(byts / ms / 1e6, 1), "unit": "GB/s",
                "ms": round(ms, 4), "bytes": byts,
                "roofline": roofline(byts / ms / 1e6, hbm, src)})
    return out


def cpu_port_baseline(hbm_unused=None):
    """The oracle's CPU SpMV (C, OpenMP over all host threads) on rows
    [0, REF_SAMPLE_ROWS) of config 5."""
    import oracle
    S = REF_SAMPLE_ROWS
    rows = oracle.synth_rowidx(SEED_A, N5, N5, OFF5, row0=0, nrows=S)
    xw = oracle.synth_vector(SEED_X, S + int(OFF5.max()))
    thr = oracle.threads()
    oracle.spmv_rowidx(OFF5, rows, rows.shape[1], xw, ncols=N5, nrows=S, nthreads=thr)
    reps = 5
    t0 = time.perf_counter()
    for _ in range(reps):
        oracle.spmv_rowidx(OFF5, rows, rows.shape[1], xw, ncols=N5, nrows=S, nthreads=thr)
    sec = (time.perf_counter() - t0) / reps
    b, _ = spmv_bytes(N5, OFF5, 0, S)
    return {"value": round(b / sec / 1e9, 2), "unit": "GB/s", "cores": thr, "kind": "port",
            "sample": f"config 5 rows [0, {S}) ({S * 27 / 1e6:.0f}M entries), mean of {reps}"}


# ------------------------------------------------------------------ arms

def setup_dist(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus and world > 1:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    if world > 1:
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return world, rank, local


PARITY_W = 132 * 1024   # rows per parity window: covers every boundary tile (max|d| = 65,793)


def spmv_window_ref(dg, w0, w1, x_full):
    """Rows [w0, w1) of the whole-matrix y = A*x, computed by the 1-GPU
    library path on a row window of A (equal to the oracle bit for bit,
    tests/test_gpu_spmv.py)."""
    Aw = dg.DiaRows.synth(N5, N5, OFF5, SEED_A, vrow0=w0, nrows=w1 - w0)
    return dg.spmv(Aw, x_full)[:w1 - w0]


def spmspm_window_ref(dg, w0, w1):
    """Rows [w0, w1) of the whole-matrix C = A*A, from row windows of A
    (rows [w0, w1)) and of B (the rows those need)."""
    d = int(OFF5.max())
    b0, b1 = max(0, w0 - d), min(N5, w1 + d)
    Aw = dg.DiaRows.synth(N5, N5, OFF5, SEED_A, vrow0=w0, nrows=w1 - w0)
    Bw = dg.DiaRows.synth(N5, N5, OFF5, SEED_A, vrow0=b0, nrows=b1 - b0)
    plan = dg.SpmspmPlan(Aw, Bw)
    Cw = plan.execute(Aw, Bw, plan.new_C())
    return plan.C_off, Cw.vals[:, :w1 - w0]


def parity_windows(r0, r1):
    """Row windows checked on a rank: both block edges (every boundary tile
    and the first interior tiles) and one window in the middle."""
    w = min(PARITY_W, r1 - r0)
    mid = (r0 + r1) // 2 // 1024 * 1024
    out = {(r0, r0 + w), (r1 - w, r1), (mid, min(r1, mid + min(w, 16384)))}
    return sorted(out)


def all_ok(flag, world):
    if world == 1:
        return flag
    t = torch.tensor([0 if flag else 1], device="cuda")
    dist.all_reduce(t)
    return int(t.item()) == 0


def emit(line):
    print(json.dumps(line, separators=(",", ":")), flush=True)


def run_ours(args):
    import diagpu_b200 as dg
    from diagpu_b200.dist import PEER, DistSpmspm, DistSpmv, Halo

    world, rank, local = setup_dist(args)
    hbm, src = peaks()
    K, W = args.steps, args.warmup
    clk = Clocks(list(range(world))) if rank == 0 else None
    if clk is not None:
        clk.__enter__()
    halo = Halo(N5, world, rank, int(OFF5.min()), int(OFF5.max()))
    r0, r1 = halo.r0, halo.r1
    A = dg.DiaRows.synth(N5, N5, OFF5, SEED_A, vrow0=r0, nrows=r1 - r0)
    ds = DistSpmv(A, halo)   # world > 1: the fused peer-halo step kernel
    dg.synth_vector(r1 - r0, SEED_X, i0=r0, out=ds.x_own)
    launches = []
    ds.step(launches)
    per_step = len(launches)
    torch.cuda.synchronize()

    # headline: K full steps (halo exchange + every row of the block)
    for _ in range(W):
        ds.step()
    barrier(world)
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(K):
        ds.step()
    e.record()
    e.synchronize()
    barrier(world)
    ms = max_over_ranks(s.elapsed_time(e) / K, world)
    total_bytes, nnz = spmv_bytes(N5, OFF5, 0, N5)
    value = total_bytes / ms / 1e6
    peer_status = ds.native.status() if ds.native is not None else 0

    # breakdown of one step: this rank's block kernel alone with no exchange
    # (back to back, and bracketed per launch for the roofline), and at N > 1
    # the NCCL forms it replaces (halo alone; halo + interior + strips)
    rank_bytes, _ = spmv_bytes(N5, OFF5, r0, r1)
    kern = lambda: dg.spmv(A, ds.x_ext, ds.y, x_lo=halo.xlo)
    kms_b2b = max_over_ranks(timed(kern, K, W, world=world), world)
    kms = max_over_ranks(timed(kern, K, W, per_launch=True), world)
    breakdown = {"step_ms": round(ms, 5), "kernel_alone_ms": round(kms_b2b, 5),
                 "kernel_alone_per_launch_ms": round(kms, 5),
                 "step_minus_kernel_ms": round(ms - kms_b2b, 5),
                 "exchange": "fused peer push (NVLink stores + step flag) inside the step kernel"
                 if world > 1 else "none (1 GPU)"}
    if world > 1:
        from diagpu_b200 import _stream, check, lib
        ds2 = DistSpmv(A, halo, native=ds.native, overlap=2)
        ds2.x_ext.copy_(ds.x_ext)
        breakdown["nccl_overlap_step_ms"] = round(
            max_over_ranks(timed(lambda: ds2.step(), K, W, world=world), world), 5)
        rg = ds.native._ranges if hasattr(ds.native, "_ranges") else halo.ranges()
        import ctypes as C

        def halo_only():
            check(lib().dia_dist_halo_start(ds.native.handle, dg._dptr(ds2.x_ext), halo.xlo, 0,
                                            1, rg.ctypes.data_as(C.c_void_p), _stream()))
            check(lib().dia_dist_halo_wait(ds.native.handle, _stream()))
        breakdown["nccl_halo_alone_ms"] = round(
            max_over_ranks(timed(halo_only, K, W, world=world), world), 5)
        del ds2

    # end to end through the public API: every step copies its x from pinned
    # host memory and its y back.  Steps are pipelined as a streaming user
    # would: step k+1's host-to-device copy and step k's device-to-host copy
    # run on their own streams (PCIe is full duplex) while SpMVs run on the
    # compute stream; double-buffered device staging, ordered by events.
    n_own = r1 - r0
    xh = torch.empty(n_own, dtype=torch.float32).pin_memory()
    xh.copy_(ds.x_own.cpu())
    yh = torch.empty(n_own, dtype=torch.float32).pin_memory()
    xst = [torch.empty(n_own, device="cuda") for _ in range(2)]
    yst = [torch.empty(n_own, device="cuda") for _ in range(2)]
    h2d, d2h = torch.cuda.Stream(), torch.cuda.Stream()
    comp = torch.cuda.current_stream()
    ev = lambda: [torch.cuda.Event() for _ in range(2)]
    in_ready, in_free, out_ready, out_free = ev(), ev(), ev(), ev()

    def e2e_run(steps, start_ev=None):
        if start_ev is not None:
            h2d.wait_event(start_ev)
            d2h.wait_event(start_ev)
        for k in range(steps):
            b = k & 1
            with torch.cuda.stream(h2d):
                h2d.wait_event(in_free[b])
                xst[b].copy_(xh, non_blocking=True)
                in_ready[b].record(h2d)
            comp.wait_event(in_ready[b])
            ds.x_own.copy_(xst[b])
            in_free[b].record(comp)
            ds.step()
            comp.wait_event(out_free[b])
            yst[b].copy_(ds.y[:n_own])
            out_ready[b].record(comp)
            with torch.cuda.stream(d2h):
                d2h.wait_event(out_ready[b])
                yh.copy_(yst[b], non_blocking=True)
                out_free[b].record(d2h)
        comp.wait_stream(d2h)
        comp.wait_stream(h2d)
    e2e_run(W)
    barrier(world)
    s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s2.record()
    e2e_run(K, s2)
    e2.record()
    e2.synchronize()
    ems = max_over_ranks(s2.elapsed_time(e2) / K, world)
    e2e_same = bool(torch.equal(yh, ds.y[:n_own].cpu()))
    peer_status |= ds.native.status() if ds.native is not None else 0

    # parity of the partitioned SpMV: this rank's rows on windows at both
    # block edges and in the middle against the whole-matrix product
    x_full = dg.synth_vector(N5, SEED_X)
    wins = parity_windows(r0, r1)
    ok_spmv = e2e_same and peer_status == 0
    for w0, w1 in wins:
        ok_spmv &= bool(torch.equal(ds.y[w0 - r0:w1 - r0], spmv_window_ref(dg, w0, w1, x_full)))
    ok_spmv = all_ok(ok_spmv, world)
    del x_full
    torch.cuda.empty_cache()

    # secondary: C = A*A on the same partitioned matrix
    if ds.native is not None:
        ds.native = None
    del ds
    if world == 1:
        B_ext = A   # one GPU: C = A*A on the matrix itself, no halo block
    else:
        B_ext = dg.DiaRows.empty(N5, N5, OFF5, vrow0=halo.xlo, nrows=halo.width, zero=True)
        B_ext.vals[:, r0 - halo.xlo:r1 - halo.xlo] = A.vals[:, :r1 - r0]
    dm = DistSpmspm(A, B_ext, halo)
    ksp = max(3, min(K, 10))
    mm_ms = max_over_ranks(timed(lambda: dm.step(), ksp, max(1, min(W, 3)), world=world), world)
    # breakdown of one partitioned C = A*A step: interior rows (own B rows
    # only), boundary rows, and at N > 1 the B halo exchange alone
    mw = max(1, min(W, 3))
    ia, ib = halo.interior()
    mm_break = {"step_ms": round(mm_ms, 4)}
    if ib > ia:
        plan_in = dm.plan_own if world > 1 else dm.plan_all
        mm_break["interior_ms"] = round(max_over_ranks(timed(
            lambda: plan_in.execute(A, dm.B, dm.C, ia, ib), ksp, mw, world=world), world), 4)
    bnd = halo.boundary()
    if world > 1:
        def bonly():
            for lo, hi in bnd:
                dm.plan_all.execute(A, dm.B, dm.C, lo, hi)
        mm_break["boundary_ms"] = round(max_over_ranks(timed(bonly, ksp, mw, world=world),
                                                       world), 4)
        if dm.native is not None:
            from diagpu_b200 import _stream, check, lib
            import ctypes as C
            rgm = halo.ranges()

            def honly():
                check(lib().dia_dist_halo_start(dm.native.handle, dg._dptr(dm.B.vals),
                                                dm.B.vrow0, dm.B.stride, dm.B.K,
                                                rgm.ctypes.data_as(C.c_void_p), _stream()))
                check(lib().dia_dist_halo_wait(dm.native.handle, _stream()))
            mm_break["halo_alone_ms"] = round(max_over_ranks(timed(honly, ksp, mw, world=world),
                                                             world), 4)
        mm_break["boundary_rows"] = sum(hi - lo for lo, hi in bnd)
    sym = dm.sym
    fl = spmspm_useful(N5, OFF5, OFF5, sym, 0, N5)
    nnzC = int(sym["C_len"].astype(np.int64).sum())
    mm_bytes = 4 * (nnz + nnzC)
    rank_mm_bytes = 4 * (nnz_rows(N5, OFF5, r0, r1) + nnz_rows(N5, sym["C_off"], r0, r1))
    del B_ext
    torch.cuda.empty_cache()
    ok_mm = True
    for w0, w1 in wins:
        c_off, Cw = spmspm_window_ref(dg, w0, w1)
        ok_mm &= bool(np.array_equal(c_off, dm.C.offsets)) and bool(
            torch.equal(dm.C.vals[:, w0 - r0:w1 - r0], Cw))
        del Cw
    ok_mm = all_ok(ok_mm, world)
    spmspm5 = {"workload": "config5 C=A*A (125 output diagonals, 729 pairs)",
               "metric": "spmspm_useful_GFLOPs", "value": round(fl / mm_ms / 1e6, 2),
               "unit": "GFLOP/s", "ms": round(mm_ms, 4), "GBps": round(mm_bytes / mm_ms / 1e6, 1),
               "bytes": mm_bytes, "useful_flops": fl, "n_gpus": world, "breakdown": mm_break,
               "roofline": roofline(rank_mm_bytes / mm_ms / 1e6, hbm, src)}
    del dm, A
    torch.cuda.empty_cache()

    extras = []
    cpu = None
    if world == 1:
        extras = single_gpu_extras(dg, K, W, hbm, src)
        if not args.no_cpu_baseline:
            ref = reference_cpu_spmv(5, 1)
            if ref is None:
                cpu = cpu_port_baseline()
            else:
                _, v_ref, thr_ref, S_ref = ref
                cpu = {"value": v_ref, "unit": "GB/s", "cores": thr_ref, "kind": "reference",
                       "sample": f"spmv_from_recon (spmv/test/test_tc_spmv.cu:64-79) on rows "
                                 f"[0, {S_ref}) of config 5 (1/16 of it), mean of 5, "
                                 f"{thr_ref} threads over row slices; a rate on the sample"}
    clocks = None
    if clk is not None:
        clk.__exit__(None, None, None)
        clocks = clk.summary()

    if rank == 0:
        for x in extras + [spmspm5]:
            emit({"secondary": x})
        rl = roofline(rank_bytes / kms / 1e6, hbm, src,
                      traffic=SPMV5_TRAFFIC if world == 1 else None)
        if world == 1:
            rl["traffic_source"] = "ncu capture of the 4,194,304-row case, scaled to a full launch"
        emit({
            "metric": "spmv_GBps", "value": round(value, 1), "unit": "GB/s", "n_gpus": world,
            "steps": K, "warmup": W, "ms_per_step": round(ms, 5), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic: counter-hash uniform[-1,1] values, seeded, generated on device",
            "config": {"workload": "config5 DIA SpMV y=A*x, 3D 27-point stencil 256x256x1024",
                       "n": N5, "diagonals": 27, "nnz": nnz, "bytes_per_step": total_bytes,
                       "parallelism": f"row-block x{world}, x halo +-65793 pushed over NVLink "
                                      "by the step kernel" if world > 1 else "1 GPU",
                       "l2": "inputs 7.8 GB > 126 MB L2 (no flush needed)"},
            "roofline": rl, "kernel_ms": round(kms, 5), "breakdown": breakdown,
            "parity": {"spmv": "bitexact" if ok_spmv else "MISMATCH",
                       "spmspm": "bitexact" if ok_mm else "MISMATCH",
                       "against": "1-GPU library product of the whole matrix on row windows",
                       "windows_per_rank": len(wins), "window_rows": PARITY_W},
            "spmspm5": {"ms": spmspm5["ms"], "GFLOPs": spmspm5["value"],
                        "frac": spmspm5["roofline"]["frac"]},
            "cpu_baseline": cpu,
            "e2e": {"value": round(total_bytes / ems / 1e6, 1), "unit": "GB/s",
                    "ms_per_step": round(ems, 4),
                    "h2d_bytes_per_step": 4 * N5, "d2h_bytes_per_step": 4 * N5,
                    "api": "diagpu_b200.dist.DistSpmv.step, pinned host x/y, steps pipelined "
                           "(H2D, SpMV, D2H on three streams)"},
            "clocks": clocks,
            "gpu_launches": per_step * K,
        })
    if world > 1:
        dist.destroy_process_group()


# ------------------------------------------------- reference GPU kernels

def _hm_structure(n, offs):
    """HM layout of a diagonal set: lengths n - |d| and prefix-sum starts."""
    offs = np.asarray(offs, np.int64)
    ln = (n - np.abs(offs)).astype(np.int64)
    st = np.concatenate([[0], np.cumsum(ln[:-1])]).astype(np.int64)
    return ln, st


def _sumset(n, a, b):
    """Ascending {da + db : |da + db| < n} (the output diagonals)."""
    s = np.unique((np.asarray(a, np.int64)[:, None] + np.asarray(b, np.int64)[None, :]).ravel())
    return s[np.abs(s) < n]


def reference_gpu_leg(steps, warmup):
    """The reference's own GPU kernels, compiled from its sources into
    oracle/_ref, timed on this GPU on the workloads the library's own arm
    times (same shapes; values from torch's seeded generator):
      tc_spmv_regdirect (spmv/src/tc_spmv_regdirect_kernel.cu:62-147) on
        config 5 in its Recon layout;
      gather_meta_kernel<512> (spmspm/spmspm.cu:256-319) and the Haque HM
        atomic kernel (spmspm/paper_hm_kernel.cu:31-93; C zeroed per launch
        as its bench does) on configs 2 and 3;
      gemm_diag_kernel (gemm_diag/gemm_diag.cu:119-329) on config 4, timed
        with its memset as gemm_diag.cu:553-566 times it.
    Each entry is one JSON line; times are mean ms per launch (CUDA events,
    back to back after warm-up)."""
    import ctypes as C

    import oracle
    torch.cuda.set_device(0)
    gen = torch.Generator(device="cuda")
    gen.manual_seed(7)
    P = lambda t: C.c_void_p(t.data_ptr())
    S = lambda: C.c_void_p(torch.cuda.current_stream().cuda_stream)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    uni = lambda shape: torch.rand(shape, generator=gen, device="cuda") * 2 - 1
    reps = max(3, min(steps, 20))
    out = []

    def tm(fn, it=reps):
        return timed(fn, it, max(1, min(warmup, 3)))

    R = oracle.ref("spmv")
    if R is not None:
        R.ref_launch_tc_spmv.argtypes = [C.c_int] * 3 + [C.c_void_p] * 3 + [C.c_int,
                                                                           C.c_void_p,
                                                                           C.c_void_p]
        n = N5
        desc = np.sort(OFF5)[::-1].astype(np.int32)
        rec = uni((len(desc), n))
        x, y = uni((n,)), torch.empty(n, device="cuda")
        doff = t(desc)
        ms = tm(lambda: R.ref_launch_tc_spmv(n, n, len(desc), P(doff), P(rec), P(x), n, P(y),
                                             S()))
        b, _ = spmv_bytes(n, OFF5, 0, n)
        out.append({"kernel": "tc_spmv_regdirect (TF32 mma.sync)",
                    "workload": "config5 SpMV, Recon layout", "ms": round(ms, 4),
                    "GBps": round(b / ms / 1e6, 1)})
        del rec, x, y
        torch.cuda.empty_cache()
    M = oracle.ref("spmspm")
    if M is not None:
        M.ref_launch_gather_meta.argtypes = ([C.c_void_p] * 4 + [C.c_int] + [C.c_void_p] * 8 +
                                             [C.c_int, C.c_int, C.c_void_p])
        M.ref_launch_hm.argtypes = ([C.c_void_p] * 4 + [C.c_int] + [C.c_void_p] * 4 + [C.c_int] +
                                    [C.c_void_p] * 4 + [C.c_int, C.c_void_p, C.c_int, C.c_int,
                                                        C.c_void_p])
        for name, n, oa, ob in (("config2 3D 7-pt 128^3 C=A*A", 128 ** 3, OFF2, OFF2),
                                ("config3 scattered 32x32 offsets n=1e6 C=A*B", 1_000_000,
                                 _scat(301), _scat(302))):
            al, ast = _hm_structure(n, oa)
            bl, bst = _hm_structure(n, ob)
            co = _sumset(n, oa, ob)
            cl, cs = _hm_structure(n, co)
            av = uni((int(al.sum()),))
            bv = av if ob is oa else uni((int(bl.sum()),))
            nnzC = int(cl.sum())
            lk = np.full(2 * n - 1, -1, np.int32)
            lk[np.asarray(ob) + n - 1] = np.arange(len(ob), dtype=np.int32)
            clk = np.full(2 * n - 1, -1, np.int32)
            clk[co + n - 1] = np.arange(len(co), dtype=np.int32)
            i32 = lambda a: t(np.asarray(a).astype(np.int32))
            dao, dbo, dco = i32(oa), i32(ob), i32(co)
            dal, dbl, dcl = i32(al), i32(bl), i32(cl)
            das, dbs, dcs = (t(np.asarray(v, np.uint64)) for v in (ast, bst, cs))
            das32, dbs32, dcs32 = i32(ast), i32(bst), i32(cs)
            dlk, dclk = t(lk), t(clk)
            Cv = torch.zeros(nnzC, device="cuda")
            gm = tm(lambda: M.ref_launch_gather_meta(P(av), P(das), P(dao), P(dal), len(oa),
                                                     P(bv), P(dbs), P(dbl), P(dlk), P(Cv),
                                                     P(dcs), P(dco), P(dcl), len(co), n, S()))
            nzA = int(al.sum())

            def hm():
                Cv.zero_()
                M.ref_launch_hm(P(av), P(dao), P(das32), P(dal), len(oa), P(bv), P(dbo),
                                P(dbs32), P(dbl), len(ob), P(Cv), P(dco), P(dcs32), P(dcl),
                                len(co), P(dclk), nzA, n, S())
            hm_ms = tm(hm)
            byts = 4 * (int(al.sum()) + (0 if ob is oa else int(bl.sum())) + nnzC)
            out.append({"kernel": "gather_meta_kernel<512>", "workload": name,
                        "ms": round(gm, 4), "GBps": round(byts / gm / 1e6, 1)})
            out.append({"kernel": "hm_structured_sparse_matmul_kernel (atomics, C zeroed)",
                        "workload": name, "ms": round(hm_ms, 4),
                        "GBps": round(byts / hm_ms / 1e6, 1)})
            del av, bv, Cv
            torch.cuda.empty_cache()
    G = oracle.ref("gemm_diag")
    if G is not None:
        G.ref_launch_gemm_diag.argtypes = ([C.c_void_p] * 4 + [C.c_int] * 3 + [C.c_void_p] * 4 +
                                           [C.c_void_p])
        n, hb = 262144, 64
        goff = np.arange(-hb, hb + 1, dtype=np.int32)
        DA, DB = uni((len(goff), n)), uni((len(goff), n))
        ks = _sumset(n, goff, goff)
        cl, cs = _hm_structure(n, ks)
        k2i = np.full(2 * n - 1, -1, np.int32)
        k2i[ks + n - 1] = np.arange(len(ks), dtype=np.int32)
        dco, dcl, dk2i, doff = t(cs.astype(np.int32)), t(cl.astype(np.int32)), t(k2i), t(goff)
        Cg = torch.zeros(int(cl.sum()), device="cuda")

        def gd():
            Cg.zero_()
            G.ref_launch_gemm_diag(P(DA), P(DB), P(doff), P(doff), len(goff), len(goff), n,
                                   P(Cg), P(dco), P(dcl), P(dk2i), S())
        ms = tm(gd, max(3, reps // 2))
        byts = 4 * (2 * nnz_rows(n, goff, 0, n) + int(cl.sum()))
        out.append({"kernel": "gemm_diag_kernel (with its memset)",
                    "workload": "config4 dense band hb=64 n=262144 gemm_diag",
                    "ms": round(ms, 4), "GBps": round(byts / ms / 1e6, 1)})
        del DA, DB, Cg
        torch.cuda.empty_cache()
    return out


def reference_cpu_spmv(steps, warmup):
    """The reference's own CPU SpMV, spmv_from_recon
    (spmv/test/test_tc_spmv.cu:64-79, compiled from the reference sources
    into oracle/_ref/), over rows [0, REF_SAMPLE_ROWS) of config 5 in the
    Recon layout, threaded over row slices.  Returns (ms per call, GB/s,
    threads, rows) or None when the library was not built."""
    import ctypes as C

    import oracle
    lib = oracle.ref("spmv")
    if lib is None:
        return None
    S = REF_SAMPLE_ROWS
    dmax = int(OFF5.max())
    rows = oracle.synth_rowidx(SEED_A, N5, N5, OFF5, row0=0, nrows=S)
    cols = S + dmax
    desc = np.sort(OFF5)[::-1].astype(np.int32)
    rec = np.zeros((len(desc), cols), np.float32)
    idx = {int(d): k for k, d in enumerate(OFF5)}
    c = np.arange(cols)
    for k, d in enumerate(desc):
        r = c - int(d)
        ok = (r >= 0) & (r < S)
        rec[k, ok] = rows[idx[int(d)], r[ok]]
    x = oracle.synth_vector(SEED_X, cols)
    y = np.zeros(S, np.float32)
    thr = oracle.threads()
    lib.ref_spmv_from_recon_threads.restype = C.c_double
    lib.ref_spmv_from_recon_threads.argtypes = [C.c_int, C.c_int, C.c_int, C.c_void_p,
                                                C.c_void_p, C.c_void_p, C.c_void_p, C.c_int,
                                                C.c_int]
    p = lambda a: a.ctypes.data_as(C.c_void_p)
    call = lambda reps: lib.ref_spmv_from_recon_threads(S, cols, len(desc), p(desc), p(rec), p(x),
                                                        p(y), thr, reps)
    if warmup:
        call(warmup)
    ms = call(steps)
    b, _ = spmv_bytes(N5, OFF5, 0, S)
    return ms, round(b / ms / 1e6, 2), thr, S


def run_reference(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    ref = reference_cpu_spmv(args.steps, args.warmup)
    if ref is None:
        print(json.dumps({"impl": "reference", "unavailable":
                          "oracle/_ref/libref_spmv.so not built (needs the reference sources)"}))
        return
    ms, v, thr, S = ref
    if world == 1 and torch.cuda.is_available() and not args.no_ref_gpu:
        for entry in reference_gpu_leg(args.steps, args.warmup):
            emit({"reference_gpu": entry})
    print(json.dumps({
        "impl": "reference", "metric": "spmv_GBps", "value": v, "unit": "GB/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 3),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic: counter-hash uniform[-1,1] values, seeded",
        "config": {"workload": "config5 DIA SpMV y=A*x, 3D 27-point stencil 256x256x1024",
                   "n": N5, "diagonals": 27},
        "cpu_baseline": {"value": v, "unit": "GB/s", "cores": thr, "kind": "reference",
                         "sample": f"spmv_from_recon (spmv/test/test_tc_spmv.cu:64-79) on rows "
                                   f"[0, {S}) of config 5, {thr} threads over row slices"},
        "e2e": {"value": v, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}),
        flush=True)


def _only_spmv(dg, n, offs):
    A = dg.DiaRows.synth(n, n, offs, SEED_A)
    x = dg.synth_vector(n, SEED_X)
    y = torch.empty(A.stride, device="cuda")
    return (lambda: dg.spmv(A, x, y)), spmv_bytes(n, offs, 0, n)[0]


def _only_spmv_block(dg, world=8, rank=1):
    """The plain block kernel on the same rank block as spmv5_peer."""
    from diagpu_b200.dist import Halo
    h = Halo(N5, world, rank, int(OFF5.min()), int(OFF5.max()))
    A = dg.DiaRows.synth(N5, N5, OFF5, SEED_A, vrow0=h.r0, nrows=h.r1 - h.r0)
    xe = dg.synth_vector(h.xhi - h.xlo, SEED_X, i0=h.xlo)
    y = torch.empty(A.stride, device="cuda")
    return (lambda: dg.spmv(A, xe, y, x_lo=h.xlo)), spmv_bytes(N5, OFF5, h.r0, h.r1)[0]


def _only_spmspm(dg, n, offsA, offsB=None, kind=0):
    A = dg.DiaRows.synth(n, n, offsA, SEED_A, kind=kind, lo=-1.0 if kind == 0 else 0.0)
    B = A if offsB is None else dg.DiaRows.synth(n, n, offsB, SEED_X, kind=kind,
                                                  lo=-1.0 if kind == 0 else 0.0)
    sym = dg.spmspm_symbolic(n, A.offsets, B.offsets)
    plan = dg.SpmspmPlan(A, B)
    Cm = plan.new_C()
    byts = 4 * (nnz_rows(n, A.offsets, 0, n) + (0 if B is A else nnz_rows(n, B.offsets, 0, n))
                + int(sym["C_len"].astype(np.int64).sum()))
    tiles = os.environ.get("DIA_BENCH_TILES", "1") == "1"
    return (lambda: plan.execute(A, B, Cm, use_tiles=tiles)), byts


def _scat(seed):
    rng = np.random.default_rng(seed)
    s = {0}
    while len(s) < 32:
        s.add(int(rng.integers(-512, 513)))
    return np.array(sorted(s), np.int32)


def _only_gemm4(dg, n=262144, hb=64, mode=0):
    goff = np.arange(-hb, hb + 1, dtype=np.int32)
    DA = dg.DiaRows.synth(n, n, goff, seed=401).vals[:, :n].contiguous()
    DB = dg.DiaRows.synth(n, n, goff, seed=402).vals[:, :n].contiguous()
    co, cl, k2i, kl, tot = dg.gemm_diag_layout(n, goff, goff)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    dco, dcl, dk2i, doff = t(co), t(cl), t(k2i), t(goff)
    C = torch.zeros(tot, device="cuda")
    fn = lambda: dg.gemm_diag(DA, DB, doff, doff, n, C, dco, dcl, dk2i, beta=0, h_off_A=goff,
                              h_off_B=goff, mode=mode)
    return fn, 4 * (2 * nnz_rows(n, goff, 0, n) + tot)


def _chain_offsets(offs, k):
    """Offsets of H^k (host sumsets; structure only)."""
    P = np.asarray(offs, np.int64)
    for _ in range(k - 1):
        P = np.unique((P[:, None] + np.asarray(offs, np.int64)[None, :]).ravel())
    return P


def chain_bytes(n, offs, k):
    """4 * (nnz(P_j) + nnz(H) + nnz(P_{j+1})) summed over the steps j = 1 .. k-1."""
    tot = 0
    for j in range(1, k):
        Pj = _chain_offsets(offs, j)
        Pj1 = _chain_offsets(offs, j + 1)
        Pj, Pj1 = Pj[np.abs(Pj) < n], Pj1[np.abs(Pj1) < n]
        tot += 4 * (nnz_rows(n, Pj, 0, n) + nnz_rows(n, offs, 0, n) + nnz_rows(n, Pj1, 0, n))
    return tot


CHAIN_K = 8
CHAIN_OFF = np.array([-1024, -1, 0, 1, 1024], np.int32)


TAYLOR_M = 16


def _only_taylor(dg, n=1 << 20, m=TAYLOR_M):
    """exp(tA) x of the config-1 operator by m chained SpMV terms."""
    A = dg.DiaRows.synth(n, n, CHAIN_OFF, seed=101, base=[-1, -1, 4, -1, -1], lo=-0.01, hi=0.01)
    x = dg.synth_vector(n, seed=102)
    y = torch.empty(n, device="cuda")
    work = torch.empty(2 * n, device="cuda")
    byts = m * 4 * (nnz_rows(n, CHAIN_OFF, 0, n) + 4 * n) + 8 * n
    return (lambda: dg.expm_taylor(A, 0.01, m, x, y, work=work)), byts


LANCZOS_M = 50


def _only_lanczos(dg, n=1 << 20, m=LANCZOS_M):
    """m Lanczos steps on the (symmetric) config-1 operator: per step a fused
    SpMV + dot, an orthogonalisation + norm, a scaling, two tiny reductions."""
    D = dg.DiaRows.empty(n, n, CHAIN_OFF)
    for k, (d, b) in enumerate(zip(CHAIN_OFF, (-1.0, -1.0, 4.0, -1.0, -1.0))):
        lo, hi = max(0, -int(d)), min(n, n - int(d))
        D.vals[k, lo:hi] = b
    x = dg.synth_vector(n, SEED_X)
    byts = m * 4 * (nnz_rows(n, CHAIN_OFF, 0, n) + 8 * n)
    return (lambda: dg.lanczos(D, m, x)), byts


def _only_spmv_c64(dg, n=256 * 256 * 256):
    """complex64 SpMV, 27-point stencil offsets on a 256^3 grid (inputs > L2)."""
    A = dg.DiaRows.empty(n, n, OFF5, dtype=torch.complex64, zero=False)
    re = dg.DiaRows.synth(n, n, OFF5, SEED_A)
    A.vals.real.copy_(re.vals)
    A.vals.imag.copy_(dg.DiaRows.synth(n, n, OFF5, SEED_A + 1).vals)
    del re
    x = torch.complex(dg.synth_vector(n, SEED_X), dg.synth_vector(n, SEED_X + 1))
    y = torch.empty(n, dtype=torch.complex64, device="cuda")
    byts = 8 * (nnz_rows(n, OFF5, 0, n) + 2 * n)
    return (lambda: dg.spmv_c64(A, x, y)), byts


def _only_chain(dg, host=False, n=1 << 20, k=CHAIN_K):
    """H^k of the config-1 operator: k-1 products P_{j+1} = P_j * H."""
    H = dg.DiaRows.synth(n, n, CHAIN_OFF, SEED_A)
    if host:
        def fn():
            P = H
            for _ in range(k - 1):
                P = dg.spmspm(P, H)
            return P
    else:
        chain = dg.PowerChain(H, max_diags=len(_chain_offsets(CHAIN_OFF, k)) + 8)

        def fn():
            chain.reset()
            for _ in range(k - 1):
                chain.step()
    return fn, chain_bytes(n, CHAIN_OFF, k)


def _only_peer(dg, world=8, rank=1):
    """The fused peer-halo step kernel on one GPU: rank `rank` of `world`
    on config 5, its neighbours emulated by local buffers and its flags set
    far ahead, so no launch waits for another (for ncu captures)."""
    import ctypes as C
    from diagpu_b200.dist import Halo, PeerHalo, spmv_rows_peer
    h = Halo(N5, world, rank, int(OFF5.min()), int(OFF5.max()))
    A = dg.DiaRows.synth(N5, N5, OFF5, SEED_A, vrow0=h.r0, nrows=h.r1 - h.r0)
    x = dg.synth_vector(N5, SEED_X)
    x_own = x[h.r0:h.r1].clone()
    rg = h.ranges()
    keep = [x_own, A]
    sh = PeerHalo()
    for q in range(2):
        lo, hi = x[h.xlo:h.r0].clone(), x[h.r1:h.xhi].clone()
        pl = torch.zeros(int(rg[3]) - h.r0, device="cuda")
        pr = torch.zeros(h.r1 - int(rg[6]), device="cuda")
        keep += [lo, hi, pl, pr]
        sh.halo_lo[q], sh.halo_hi[q] = lo.data_ptr(), hi.data_ptr()
        sh.peer_left_halo_hi[q], sh.peer_right_halo_lo[q] = pl.data_ptr(), pr.data_ptr()
    ctl = torch.zeros(8, dtype=torch.int64, device="cuda")
    ctl[0] = ctl[1] = 1 << 40
    pctl = torch.zeros(2, dtype=torch.int64, device="cuda")
    keep += [ctl, pctl]
    sh.flag_lo, sh.flag_hi = ctl.data_ptr(), ctl.data_ptr() + 8
    sh.push_count, sh.status = ctl.data_ptr() + 16, ctl.data_ptr() + 32
    sh.peer_left_flag_hi, sh.peer_right_flag_lo = pctl.data_ptr() + 8, pctl.data_ptr()
    sh.send_left_hi, sh.send_right_lo = int(rg[3]), int(rg[6])
    sh.has_left, sh.has_right = 1, 1
    sh.timeout_ns = 2_000_000_000
    y = torch.empty(A.stride, device="cuda")
    step = [0]

    def fn():
        step[0] += 1
        spmv_rows_peer(sh, step[0], A, h.r0, h.r1, h.xlo, h.xhi, x_own, y)
    fn.keep = keep
    return fn, spmv_bytes(N5, OFF5, h.r0, h.r1)[0]


# name -> builder(dg) returning (callable, algorithmic bytes); the "_s" cases
# are reduced sizes (<= a few GB on the device) for ncu captures
ONLY = {
    "spmv5": lambda dg: _only_spmv(dg, N5, OFF5),
    "spmv5_s": lambda dg: _only_spmv(dg, 256 * 256 * 64, OFF5),
    "spmv1": lambda dg: _only_spmv(dg, 1 << 20, np.array([-1024, -1, 0, 1, 1024], np.int32)),
    "spmv5_peer": lambda dg: _only_peer(dg),
    "spmv5_block8": lambda dg: _only_spmv_block(dg),
    "spmspm5": lambda dg: _only_spmspm(dg, N5, OFF5),
    "spmspm5_s": lambda dg: _only_spmspm(dg, 256 * 256 * 64, OFF5),
    "spmspm2": lambda dg: _only_spmspm(dg, 128 ** 3, np.array([-16384, -128, -1, 0, 1, 128,
                                                                16384], np.int32)),
    "spmspm3": lambda dg: _only_spmspm(dg, 1_000_000, _scat(301), _scat(302), kind=1),
    "gemm4": lambda dg: _only_gemm4(dg),
    "chain1": lambda dg: _only_chain(dg),
    "taylor1": lambda dg: _only_taylor(dg),
    "spmvc": lambda dg: _only_spmv_c64(dg),
    "lanczos1": lambda dg: _only_lanczos(dg),
    "chain1_host": lambda dg: _only_chain(dg, host=True),
    "gemm4_simt": lambda dg: _only_gemm4(dg, mode=1),
}


def run_only(args):
    import diagpu_b200 as dg
    torch.cuda.set_device(0)
    fn, byts = ONLY[args.only](dg)
    ms = timed(fn, args.steps, args.warmup)
    print(json.dumps({"only": args.only, "ms": round(ms, 4), "bytes": byts,
                      "GBps": round(byts / ms / 1e6, 1)}), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-ref-gpu", action="store_true",
                    help="reference arm: skip the reference's GPU kernels")
    ap.add_argument("--only", choices=sorted(ONLY), default=None,
                    help="run one workload `steps` times (for profiling) and print its time")
    args = ap.parse_args()
    if args.only:
        return run_only(args)
    if args.warmup < 3 and args.impl == "ours":
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
