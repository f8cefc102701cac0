"""Build libdiagpu_b200.so in-tree for sm_100a (nvcc cross-compiles; no GPU
needed).  Usage: python -m diagpu_b200._build  (or __graft_entry__.build()).
"""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libdiagpu_b200.so")
SOURCES = ["status.cu", "spmv.cu", "spmspm.cu", "spmspm_tiled.cu", "spmspm_runpair.cu", "symbolic.cu", "gemm_diag.cu",
           "gemm_diag_tc.cu", "synth.cu", "dist.cu", "dist_peer.cu", "chain.cu", "io_mtx.cu", "krylov.cu", "io_pauli.cu"]
NVCC = os.environ.get("NVCC", "nvcc")
FLAGS = ["-O3", "-std=c++17", "-gencode", "arch=compute_100a,code=sm_100a", "-lineinfo",
         "-Xcompiler", "-fPIC", "-Xptxas", "-O3", "--expt-relaxed-constexpr",
         "-ccbin", "/usr/bin/g++"]


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(verbose: bool = False, force: bool = False) -> str:
    objdir = os.path.join(HERE, "_build")
    os.makedirs(objdir, exist_ok=True)
    headers = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    headers += [os.path.join(ROOT, "include", f) for f in os.listdir(os.path.join(ROOT, "include"))]
    objs = []
    for src in SOURCES:
        s = os.path.join(CSRC, src)
        o = os.path.join(objdir, src + ".o")
        objs.append(o)
        if force or _stale(o, [s] + headers):
            cmd = [NVCC, *FLAGS, "-c", s, "-o", o, "-I", os.path.join(ROOT, "include")]
            if verbose:
                print(" ".join(cmd), flush=True)
            subprocess.run(cmd, check=True)
    if force or _stale(LIB, objs):
        cmd = [NVCC, "-shared", "-gencode", "arch=compute_100a,code=sm_100a", "-ccbin",
               "/usr/bin/g++", *objs, "-o", LIB, "-lnccl"]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    print(build(verbose=True, force="--force" in sys.argv))
