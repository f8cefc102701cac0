"""The reference's own SpMV test and benchmark, unmodified, linked against
libdiagpu_b200.so instead of the reference kernel (oracle/Makefile builds
them into oracle/_ref where the reference sources exist): the C++ drop-in
check of launch_tc_spmv_regdirect.  The reference programs verify the
launcher's y against their CPU references (TF32 tolerance 1e-2, which the
FP32 library meets with room to spare)."""
import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.path.join(ROOT, "oracle", "_ref")

pytestmark = pytest.mark.gpu


def _run(name, args=(), ok_text=""):
    exe = os.path.join(REF, name)
    if not os.path.exists(exe):
        pytest.skip(f"{name} not built (needs the reference sources at build time)")
    p = subprocess.run([exe, *args], capture_output=True, text=True, timeout=600)
    assert p.returncode == 0, p.stdout[-2000:] + p.stderr[-2000:]
    assert ok_text in p.stdout, p.stdout[-2000:]
    return p.stdout


def test_reference_test_tc_spmv_links_and_passes():
    out = _run("test_tc_spmv_dropin", ok_text="ALL TESTS PASSED")
    assert out.count("[OK]") == 6


def test_reference_bench_cusparse_links_and_verifies():
    _run("bench_cusparse_dropin", ["262144"], ok_text="RESULTS VERIFIED")
