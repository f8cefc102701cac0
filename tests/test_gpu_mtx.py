"""A Matrix Market file from the reference's generator, ingested with
read_mtx, drives the GPU SpMV: equal bit for bit to the reference's CPU CSR
loop (orc_spmv_csr, spmv/bench/bench_cusparse.cu:119-126) on the CSR that
scipy reads from the same file."""
import os
import warnings

import numpy as np
import pytest
import scipy.io as sio

import diagpu_b200 as dg
import oracle
from tests._util import same

pytestmark = pytest.mark.gpu


def test_spmv_on_ingested_reference_file():
    path = os.path.join(os.path.dirname(__file__), "golden", "banded_64.mtx")
    A = dg.read_mtx(path)
    with warnings.catch_warnings():
        warnings.simplefilter("ignore")
        S = sio.mmread(path).tocsr()
    S.sort_indices()
    x = dg.synth_vector(A.n_cols, seed=7)
    y = dg.spmv(A, x)[:A.n_rows].cpu().numpy()
    ref = oracle.spmv_csr(A.n_rows, S.indptr.astype(np.int32), S.indices.astype(np.int32),
                          S.data.astype(np.float32), x.cpu().numpy())
    assert same(y, ref)
