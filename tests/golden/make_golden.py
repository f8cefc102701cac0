"""Generate the golden fixtures in tests/golden/ from the reference itself.

Run where the reference sources exist (they are not on the GPU box):

    make -C oracle            # builds oracle/_ref/libref_*.so from the sources
    python tests/golden/make_golden.py

Every output array below comes from a reference routine compiled from the
reference's own sources (oracle/ref/*.cu shims); the script only chooses
inputs and stores results.  Inputs follow the reference's own test and
benchmark generators:

  spmv_kat5.npz      the 5x5 known-answer matrix and x = 1..5 of
                     spmv/test/test_reconstruct.cpp:185-193 (parsed from that
                     file), through dense_to_dia / build_recon /
                     spmv_from_recon.
  spmv_cases.npz     the six structures of spmv/test/test_tc_spmv.cu:168-179,
                     data from that test's LCG (:87-98).
  spmspm_banded.npz  make_banded(n, w, 1234/5678) of
                     spmspm/bench_spmspm.cu:89-106,465-466 at small n;
                     make_c_structure, cpu_dia_spgemm, dense_ref_to_cdiag.
  spmspm_scatter.npz 32 scattered offsets per operand in [-512, 512] incl. 0
                     (the shape of the scattered SpMSpM config), values from
                     numpy; cpu_dia_spgemm + compute_c_hm_structure.
  gemm_diag.npz      pack_diag_matrix(n, -hb..hb, 42/137) of
                     gemm_diag/gemm_diag.cu:361-382,485-486; build_c_layout;
                     cpu_diag_multiply (dense, mapped to the HM layout).
  banded_64.mtx      the Matrix Market file spmv/tools/gen_banded_mtx.cpp
                     writes for n = 64 (its SpMV benchmark's banded matrix),
                     from the generator compiled unmodified into
                     oracle/_ref/gen_banded_mtx.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
import re
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
import oracle  # noqa: E402

REF = os.environ.get("DIAGPU_REFERENCE", "/root/reference")
OUT = os.path.dirname(os.path.abspath(__file__))


def P(a, dt):
    a = np.ascontiguousarray(a, dtype=dt)
    return a, a.ctypes.data_as(C.c_void_p)


def ref_dense_to_dia(lib, H):
    rows, cols = H.shape
    cap = rows + cols - 1
    off = np.zeros(cap, np.int32)
    st = np.zeros(cap, np.int32)
    ln = np.zeros(cap, np.int32)
    val = np.zeros(rows * cols, np.float32)
    nv = C.c_int(0)
    Hc = np.ascontiguousarray(H, np.float32)
    K = lib.ref_dense_to_dia(Hc.ctypes.data_as(C.c_void_p), rows, cols,
                             off.ctypes.data_as(C.c_void_p), st.ctypes.data_as(C.c_void_p),
                             ln.ctypes.data_as(C.c_void_p), val.ctypes.data_as(C.c_void_p),
                             C.byref(nv))
    return off[:K].copy(), st[:K].copy(), ln[:K].copy(), val[:nv.value].copy()


def ref_recon_and_spmv(lib, rows, cols, dia, x):
    off, st, ln, val = dia
    K = len(off)
    roff = np.zeros(K, np.int32)
    rval = np.zeros(K * cols, np.float32)
    _, po = P(off, np.int32)
    lib.ref_build_recon(rows, cols, K, off.ctypes.data_as(C.c_void_p),
                        st.ctypes.data_as(C.c_void_p), ln.ctypes.data_as(C.c_void_p),
                        val.ctypes.data_as(C.c_void_p), len(val),
                        roff.ctypes.data_as(C.c_void_p), rval.ctypes.data_as(C.c_void_p))
    y = np.zeros(rows, np.float32)
    xc = np.ascontiguousarray(x, np.float32)
    lib.ref_spmv_from_recon(rows, cols, K, roff.ctypes.data_as(C.c_void_p),
                            rval.ctypes.data_as(C.c_void_p), xc.ctypes.data_as(C.c_void_p),
                            y.ctypes.data_as(C.c_void_p))
    return roff, rval.reshape(K, cols), y


def kat5(lib):
    src = open(os.path.join(REF, "spmv/test/test_reconstruct.cpp")).read()
    m = re.search(r"float\s+H_dense\[N \* N\]\s*=\s*\{([^}]*)\}", src)
    H = np.array([float(t) for t in m.group(1).replace("\n", " ").split(",") if t.strip()],
                 np.float32).reshape(5, 5)
    m = re.search(r"float\s+x_arr\[N\]\s*=\s*\{([^}]*)\}", src)
    x = np.array([float(t) for t in m.group(1).split(",") if t.strip()], np.float32)
    dia = ref_dense_to_dia(lib, H)
    roff, rval, y = ref_recon_and_spmv(lib, 5, 5, dia, x)
    np.savez(os.path.join(OUT, "spmv_kat5.npz"), H=H, x=x, dia_off=dia[0], dia_start=dia[1],
             dia_len=dia[2], dia_val=dia[3], recon_off=roff, recon=rval, y=y,
             y_dense=(H.astype(np.float64) @ x.astype(np.float64)).astype(np.float32))


def lcg_case(N, offsets):
    """Data generator of spmv/test/test_tc_spmv.cu:85-98 (seeded LCG)."""
    seed = (0x1234567 + N) & 0xFFFFFFFF

    def rng():
        nonlocal seed
        seed = (seed * 1664525 + 1013904223) & 0xFFFFFFFF
        return np.float32(((seed >> 8) & 0xFFFF) / 65536.0 * 2.0 - 1.0)

    H = np.zeros((N, N), np.float32)
    for r in range(N):
        for d in offsets:
            c = r + d
            if 0 <= c < N:
                H[r, c] = rng()
    x = np.array([rng() for _ in range(N)], np.float32)
    return H, x


def spmv_cases(lib):
    cases = [("tridiagonal", 48, [-1, 0, 1]), ("tridiag_ragged", 37, [-1, 0, 1]),
             ("pentadiagonal", 64, [-2, -1, 0, 1, 2]),
             ("wide9", 80, [-9, -5, -2, -1, 0, 1, 2, 5, 9]),
             ("asymmetric", 71, [-3, 0, 2, 4, 7]), ("main_only", 16, [0])]
    out = {}
    for name, N, offs in cases:
        H, x = lcg_case(N, offs)
        dia = ref_dense_to_dia(lib, H)
        roff, rval, y = ref_recon_and_spmv(lib, N, N, dia, x)
        out[f"{name}__H"] = H
        out[f"{name}__x"] = x
        out[f"{name}__recon_off"] = roff
        out[f"{name}__recon"] = rval
        out[f"{name}__y"] = y
    np.savez(os.path.join(OUT, "spmv_cases.npz"), names=np.array([c[0] for c in cases]), **out)


def ref_spmspm(lib, n, A, B):
    Ao, Al, As, Av = A
    Bo, Bl, Bs, Bv = B
    cap = len(Ao) * len(Bo) + 1
    Co = np.zeros(cap, np.int32)
    Cl = np.zeros(cap, np.int32)
    Cs = np.zeros(cap, np.int64)
    ptr = lambda a: a.ctypes.data_as(C.c_void_p)
    nC = lib.ref_make_c_structure(n, len(Ao), ptr(Ao), len(Bo), ptr(Bo), ptr(Co), ptr(Cl), ptr(Cs))
    Co, Cl, Cs = Co[:nC].copy(), Cl[:nC].copy(), Cs[:nC].copy()
    nnz = int(Cs[-1] + Cl[-1]) if nC else 0
    Cv = np.zeros(max(nnz, 1), np.float32)
    lib.ref_cpu_dia_spgemm(n, len(Ao), ptr(Ao), ptr(Al), ptr(As), ptr(Av), len(Bo), ptr(Bo),
                           ptr(Bl), ptr(Bs), ptr(Bv), nC, ptr(Co), ptr(Cl), ptr(Cs), ptr(Cv))
    # the Haque baseline's own symbolic phase must agree
    ho = np.zeros(cap, np.int32)
    hl = np.zeros(cap, np.int32)
    hs = np.zeros(cap, np.int32)
    nH = lib.ref_compute_c_hm_structure(n, len(Ao), ptr(Ao), len(Bo), ptr(Bo), ptr(ho), ptr(hl),
                                        ptr(hs))
    assert nH == nC and (ho[:nC] == Co).all() and (hl[:nC] == Cl).all() and (hs[:nC] == Cs).all()
    return Co, Cl, Cs, Cv[:nnz]


def make_banded(lib, n, w, seed):
    K = 2 * w + 1
    off = np.zeros(K, np.int32)
    ln = np.zeros(K, np.int32)
    st = np.zeros(K, np.int64)
    ptr = lambda a: a.ctypes.data_as(C.c_void_p)
    nnz = lib.ref_make_banded(n, w, C.c_uint(seed), ptr(off), ptr(ln), ptr(st), None)
    val = np.zeros(max(nnz, 1), np.float32)
    lib.ref_make_banded(n, w, C.c_uint(seed), ptr(off), ptr(ln), ptr(st), ptr(val))
    keep = np.arange(sum(1 for d in range(-w, w + 1) if n - abs(d) > 0))
    return off[keep].copy(), ln[keep].copy(), st[keep].copy(), val[:nnz].copy()


def spmspm_banded(lib):
    out = {}
    cases = [("n1000_w16", 1000, 16), ("n257_w3", 257, 3), ("n20_w16", 20, 16), ("n1_w2", 1, 2)]
    ptr = lambda a: a.ctypes.data_as(C.c_void_p)
    for name, n, w in cases:
        A = make_banded(lib, n, w, 1234)
        B = make_banded(lib, n, w, 5678)
        Co, Cl, Cs, Cv = ref_spmspm(lib, n, A, B)
        for tag, M in (("A", A), ("B", B)):
            for f, v in zip(("off", "len", "start", "val"), M):
                out[f"{name}__{tag}_{f}"] = v
        out[f"{name}__C_off"], out[f"{name}__C_len"] = Co, Cl
        out[f"{name}__C_start"], out[f"{name}__C_val"] = Cs, Cv
        if n <= 1000:
            dense = np.zeros(max(len(Cv), 1), np.float32)
            Ao, Al, As, Av = A
            Bo, Bl, Bs, Bv = B
            lib.ref_dense_ref_to_cdiag(n, len(Ao), ptr(Ao), ptr(Al), ptr(As), ptr(Av), len(Bo),
                                       ptr(Bo), ptr(Bl), ptr(Bs), ptr(Bv), len(Co), ptr(Co),
                                       ptr(Cl), ptr(Cs), ptr(dense))
            out[f"{name}__C_dense"] = dense[: len(Cv)]
    np.savez(os.path.join(OUT, "spmspm_banded.npz"), names=np.array([c[0] for c in cases]),
             **out)


def spmspm_scatter(lib):
    rng = np.random.default_rng(20261201)
    out = {}
    cases = [("n1100_k16", 1100, 16), ("n600_k32", 600, 32), ("n64_k8", 64, 8)]
    for name, n, k in cases:
        mats = []
        for _ in range(2):
            offs = {0}
            while len(offs) < k:
                offs.add(int(rng.integers(-512, 513)))
            offs = np.array(sorted(o for o in offs if abs(o) < n), np.int32)
            ln = (n - np.abs(offs)).astype(np.int32)
            st = np.concatenate([[0], np.cumsum(ln[:-1], dtype=np.int64)]).astype(np.int64)
            val = rng.standard_normal(int(ln.sum())).astype(np.float32)
            mats.append((offs, ln, st, val))
        A, B = mats
        Co, Cl, Cs, Cv = ref_spmspm(lib, n, A, B)
        for tag, M in (("A", A), ("B", B)):
            for f, v in zip(("off", "len", "start", "val"), M):
                out[f"{name}__{tag}_{f}"] = v
        out[f"{name}__C_off"], out[f"{name}__C_len"] = Co, Cl
        out[f"{name}__C_start"], out[f"{name}__C_val"] = Cs, Cv
    np.savez(os.path.join(OUT, "spmspm_scatter.npz"), names=np.array([c[0] for c in cases]),
             **out)


def gemm_diag(lib):
    out = {}
    cases = [("n256_hb10", 256, 10), ("n300_hb4", 300, 4), ("n128_hb64", 128, 64)]
    ptr = lambda a: a.ctypes.data_as(C.c_void_p)
    for name, n, hb in cases:
        offs = np.arange(-hb, hb + 1, dtype=np.int32)
        P_ = len(offs)
        DA = np.zeros(P_ * n, np.float32)
        DB = np.zeros(P_ * n, np.float32)
        lib.ref_pack_diag_matrix(n, P_, ptr(offs), C.c_uint(42), ptr(DA))
        lib.ref_pack_diag_matrix(n, P_, ptr(offs), C.c_uint(137), ptr(DB))
        cap = 2 * n - 1
        co = np.zeros(cap, np.int32)
        cl = np.zeros(cap, np.int32)
        k2i = np.zeros(cap, np.int32)
        kl = np.zeros(cap, np.int32)
        tot = C.c_int(0)
        nk = lib.ref_build_c_layout(n, P_, ptr(offs), P_, ptr(offs), ptr(co), ptr(cl), ptr(k2i),
                                    ptr(kl), C.byref(tot))
        dense = np.zeros(n * n, np.float32)
        lib.ref_cpu_diag_multiply(ptr(DA), ptr(offs), P_, ptr(DB), ptr(offs), P_, n, ptr(dense))
        dense = dense.reshape(n, n)
        C_hm = np.zeros(tot.value, np.float32)
        for ki in range(nk):
            k = kl[ki]
            sr, sc = (0, k) if k >= 0 else (-k, 0)
            p = np.arange(cl[ki])
            C_hm[co[ki] + p] = dense[sr + p, sc + p]
        out.update({f"{name}__off": offs, f"{name}__DA": DA, f"{name}__DB": DB,
                    f"{name}__C_offsets": co[:nk].copy(), f"{name}__C_lens": cl[:nk].copy(),
                    f"{name}__k_to_idx": k2i.copy(), f"{name}__k_list": kl[:nk].copy(),
                    f"{name}__C": C_hm})
    np.savez(os.path.join(OUT, "gemm_diag.npz"), names=np.array([c[0] for c in cases]), **out)


def banded_mtx(n=64):
    """The reference's gen_banded_mtx output (Matrix Market text) for n rows."""
    exe = os.path.join(os.path.dirname(oracle.__file__), "_ref", "gen_banded_mtx")
    path = os.path.join(OUT, f"banded_{n}.mtx")
    subprocess.run([exe, str(n), path], check=True, capture_output=True)


def main():
    s = oracle.ref("spmv")
    m = oracle.ref("spmspm")
    g = oracle.ref("gemm_diag")
    if s is None or m is None or g is None:
        raise SystemExit("oracle/_ref not built: run `make -C oracle` where the reference exists")
    m.ref_make_banded.restype = C.c_longlong
    kat5(s)
    spmv_cases(s)
    spmspm_banded(m)
    spmspm_scatter(m)
    gemm_diag(g)
    banded_mtx()
    for f in sorted(os.listdir(OUT)):
        if f.endswith((".npz", ".mtx")):
            print(f, os.path.getsize(os.path.join(OUT, f)))


if __name__ == "__main__":
    main()
