"""Pauli-string Hamiltonians through the GPU paths: a transverse-field Ising
chain's ground-state energy from the device Lanczos against dense
eigenvalues, and a complex sum's SpMV and exp(-iHt) against dense numpy."""
import numpy as np
import pytest
import scipy.linalg as sl
import torch

import diagpu_b200 as dg
from tests.test_pauli import dense, random_terms

pytestmark = pytest.mark.gpu


def test_ising_ground_energy_by_lanczos():
    nq = 10
    terms = ([(-1.0, f"Z{k} Z{k + 1}") for k in range(nq - 1)] +
             [(-0.7, f"X{k}") for k in range(nq)])
    H = dg.pauli_to_dia(terms, nq)                     # real: float32 DiaRows
    assert H.vals.dtype == torch.float32
    x = dg.synth_vector(H.n_rows, seed=3)
    al, be = dg.lanczos(H, 80, x)
    a, b = al.cpu().numpy(), be.cpu().numpy()
    T = np.diag(a) + np.diag(b[:-1], 1) + np.diag(b[:-1], -1)
    e0 = np.linalg.eigvalsh(T).min()
    ref = np.linalg.eigvalsh(dense(terms, nq).real).min()
    assert abs(e0 - ref) / abs(ref) < 1e-5


def test_complex_hamiltonian_spmv_and_evolution():
    nq = 9
    terms = random_terms(np.random.default_rng(7), nq, 30, complex_coef=False)
    Hd = dense(terms, nq)
    H = dg.pauli_to_dia(terms, nq, real=False)
    assert H.vals.dtype == torch.complex64
    rng = np.random.default_rng(8)
    x = (rng.standard_normal(H.n_rows) + 1j * rng.standard_normal(H.n_rows)).astype(np.complex64)
    y = dg.spmv_c64(H, torch.from_numpy(x).cuda()).cpu().numpy()
    ref = Hd @ x.astype(np.complex128)
    assert np.linalg.norm(y - ref) / np.linalg.norm(ref) < 1e-6
    # Hermitian (real coefficients, Pauli strings are Hermitian): unitary evolution
    t = 0.05
    yt = dg.expm_taylor_c64(H, t, 24, torch.from_numpy(x).cuda()).cpu().numpy()
    reft = sl.expm(-1j * t * Hd) @ x.astype(np.complex128)
    assert np.linalg.norm(yt - reft) / np.linalg.norm(reft) < 1e-5
