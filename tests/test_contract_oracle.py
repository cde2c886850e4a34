"""The fused multiply-add fold (BST_PROGRAM_CONTRACT) in the C oracle, pinned on the CPU.

* Every later multiplied term must fold as ONE correctly rounded a*b + c.  An independent
  restatement with exact rational arithmetic (fractions.Fraction, whose conversion to float
  rounds to nearest-even) checks the C oracle's fma/fmaf fold point by point (fp64).
* Contraction changes rounding only: against the separately rounded fold the normwise
  relative difference stays below the tolerances the path is held to (1e-6 fp32,
  1e-12 fp64), and single-term programs are unchanged.
"""
from fractions import Fraction

import numpy as np
import pytest

import oracle
from basalto import program as P
from basalto import workloads as W
from conftest import oracle_terms


def _exact_contracted_f64(x, terms, init_zero):
    """Point-by-point fold with the fused terms computed exactly, then rounded once."""
    out = np.empty_like(x)
    n = x.shape
    for idx in np.ndindex(*n):
        acc = 0.0
        for g, (op, sc, taps) in enumerate(terms):
            s = 0.0
            for j, o in enumerate(taps):
                q = tuple(i + d for i, d in zip(idx, o))
                v = float(x[q]) if all(0 <= a < b for a, b in zip(q, n)) else 0.0
                s = v if j == 0 else s + v
            c = float(sc)
            if g == 0:
                t = c * s if op == "mul" else (s / c if op == "div" else s)
                acc = 0.0 + t if init_zero else t
            elif op == "mul":
                acc = float(Fraction(c) * Fraction(s) + Fraction(acc))
            else:
                acc = acc + (s / c if op == "div" else s)
        out[idx] = acc
    return out


@pytest.mark.parametrize("prog", [P.box(3, 1, W.box27_weights()), P.heat7_3d(), P.star_3d(P.LAPLACIAN8_COEFFS)])
def test_c_oracle_fma_fold_is_exactly_rounded(prog):
    x = np.random.default_rng(3).standard_normal((5, 6, 7))
    terms = oracle_terms(prog)
    got = oracle.program_c(x, terms, init_zero=prog.init_zero, contract=True)
    ref = _exact_contracted_f64(x, terms, prog.init_zero)
    assert np.array_equal(got, ref)


@pytest.mark.parametrize("dtype,tol", [(np.float32, 1e-6), (np.float64, 1e-12)])
def test_contraction_changes_rounding_only(dtype, tol):
    rng = np.random.default_rng(11)
    for prog in (P.box(3, 1, W.box27_weights()), P.heat7_3d(), P.star_3d(P.LAPLACIAN8_COEFFS)):
        x = rng.standard_normal((16, 17, 18)).astype(dtype)
        terms = oracle_terms(prog)
        a = oracle.program_c(x, terms, init_zero=prog.init_zero)
        b = oracle.program_c(x, terms, init_zero=prog.init_zero, contract=True)
        assert not np.array_equal(a, b)  # the fold really differs
        assert np.abs(a - b).max() / np.abs(a).max() < tol
    j = P.jacobi5_2d()  # one multiplied term: nothing to fuse
    x = rng.standard_normal((20, 24)).astype(dtype)
    assert np.array_equal(oracle.program_c(x, oracle_terms(j)), oracle.program_c(x, oracle_terms(j), contract=True))


def test_program_flag_round_trip():
    from basalto import _abi
    p = P.heat7_3d()
    assert p.to_c((4, 4, 4)).flags == 0
    q = p.contracted()
    assert q.contract and q.to_c((4, 4, 4)).flags == _abi.BST_PROGRAM_CONTRACT
    assert q.pack((4, 4, 4)) != p.pack((4, 4, 4))  # the interceptor's plan key sees the flag
    assert q.contracted(False) == p
