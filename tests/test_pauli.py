"""Pauli-string Hamiltonians into DIA (dia_pauli_to_dia, host side: no GPU).

Checked entry for entry against the dense operator built from Kronecker
products of the 2x2 Pauli matrices (numpy), with qubit k on bit k of the
basis index: the convention of the reference's talk, where an X or Y on
qubit k moves the column by +-2^k."""
import numpy as np
import pytest

import diagpu_b200 as dg

PAULI = {"I": np.eye(2), "X": np.array([[0, 1], [1, 0]]),
         "Y": np.array([[0, -1j], [1j, 0]]), "Z": np.diag([1, -1])}


def dense(terms, nq, big_endian=False):
    H = np.zeros((1 << nq, 1 << nq), np.complex128)
    for coef, ops in terms:
        per = ["I"] * nq
        for op in ops.split():
            per[int(op[1:])] = op[0]
        # qubit k on bit k: the most significant factor is qubit nq-1
        order = per if big_endian else per[::-1]
        M = np.array([[1.0 + 0j]])
        for p in order:
            M = np.kron(M, PAULI[p])
        H += complex(coef) * M
    return H


def from_dia(n, offs, vals):
    A = np.zeros((n, n), np.complex64)
    for k, d in enumerate(offs):
        for r in range(n):
            c = r + int(d)
            if 0 <= c < n:
                A[r, c] = vals[k, r]
            else:
                assert vals[k, r] == 0
        assert (vals[k, n:] == 0).all()
    return A


def random_terms(rng, nq, nterms, complex_coef):
    terms = []
    for _ in range(nterms):
        ops = [f"{'XYZ'[rng.integers(3)]}{q}" for q in range(nq) if rng.random() < 0.35]
        c = rng.standard_normal() + (1j * rng.standard_normal() if complex_coef else 0)
        terms.append((c, " ".join(ops)))
    return terms


@pytest.mark.parametrize("nq,nterms,cplx", [(1, 3, False), (3, 10, True), (5, 25, False),
                                            (6, 40, True)])
def test_random_pauli_sums_match_dense(nq, nterms, cplx):
    rng = np.random.default_rng(nq * 100 + nterms)
    terms = random_terms(rng, nq, nterms, cplx)
    n, offs, vals, real = dg.pauli_to_dia_host(terms, nq)
    assert n == 1 << nq and np.all(np.diff(offs) > 0)
    ref = dense(terms, nq).astype(np.complex64)
    assert np.array_equal(from_dia(n, offs, vals), ref)
    assert real == bool(np.all(ref.imag == 0))


def test_big_endian_ordering_matches_openfermion_convention():
    terms = [(0.7, "X0 Z2"), (-0.3, "Y1 Y3"), (1.1, "Z0 Z1")]
    n, offs, vals, _ = dg.pauli_to_dia_host(terms, 4, big_endian=True)
    assert np.array_equal(from_dia(n, offs, vals), dense(terms, 4, big_endian=True).astype(np.complex64))


def test_transverse_field_ising_is_real_and_banded():
    """H = -J sum Z_k Z_{k+1} - h sum X_k: real, on the offsets 0 and +-2^k."""
    nq = 8
    terms = [(-1.0, f"Z{k} Z{k + 1}") for k in range(nq - 1)] + [(-0.6, f"X{k}") for k in range(nq)]
    n, offs, vals, real = dg.pauli_to_dia_host(terms, nq)
    assert real
    assert sorted(offs.tolist()) == sorted([0] + [s * (1 << k) for k in range(nq) for s in (1, -1)])
    ref = dense(terms, nq).astype(np.complex64)
    assert np.array_equal(from_dia(n, offs, vals), ref)


def test_qubit_operator_text():
    text = "0.5 [X0 Y1] +\n(-0.25+0.1j) [Z2] +\n1.0 []"
    terms = dg.parse_pauli_sum(text)
    assert terms == [(0.5 + 0j, "X0 Y1"), (-0.25 + 0.1j, "Z2"), (1 + 0j, "")]
    n, offs, vals, real = dg.pauli_to_dia_host(text)
    assert n == 8 and not real
    assert np.array_equal(from_dia(n, offs, vals), dense(terms, 3).astype(np.complex64))


def test_errors():
    with pytest.raises(dg.DiaError):
        dg.pauli_to_dia_host([(1.0, "X3")], 2)        # qubit beyond nq
    with pytest.raises(dg.DiaError):
        dg.pauli_to_dia_host([(1.0, "Q0")], 2)        # not a Pauli operator
    with pytest.raises(dg.DiaError) as e:             # 2^17 diagonals: not banded
        dg.pauli_to_dia_host([(1.0, " ".join(f"X{k}" for k in range(17)))], 17)
    assert e.value.code == dg.DIA_ERR_UNSUPPORTED


def test_wide_strings_rejected_without_enumerating():
    """A 30-qubit all-X string spans 2^30 diagonals: rejected at once with
    DIA_ERR_UNSUPPORTED (no multi-GiB offset list is built first)."""
    import time
    t0 = time.perf_counter()
    with pytest.raises(dg.DiaError) as e:
        dg.pauli_to_dia_host([(1.0, " ".join(f"X{q}" for q in range(30)))], 30)
    assert e.value.code == dg.DIA_ERR_UNSUPPORTED
    assert time.perf_counter() - t0 < 5.0


def test_many_sixteen_x_strings_stop_at_the_cap():
    """Each string has 16 X factors (65536 diagonals, allowed alone); their
    union passes 65536 and the call stops with DIA_ERR_UNSUPPORTED."""
    terms = [(1.0, " ".join(f"X{q}" for q in range(s, s + 16))) for s in range(8)]
    with pytest.raises(dg.DiaError) as e:
        dg.pauli_to_dia_host(terms, 24)
    assert e.value.code == dg.DIA_ERR_UNSUPPORTED


def test_terms_sharing_an_x_mask_share_tables():
    """Many terms on one X mask with different Z masks: still exact."""
    rng = np.random.default_rng(7)
    terms = []
    for _ in range(30):
        zs = [f"Z{q}" for q in (2, 3, 4) if rng.random() < 0.5]
        terms.append((rng.standard_normal(), " ".join(["X0", "Y1"] + zs)))
    n, offs, vals, real = dg.pauli_to_dia_host(terms, 5)
    ref = dense(terms, 5).astype(np.complex64)
    assert np.allclose(from_dia(n, offs, vals), ref, atol=1e-5)
