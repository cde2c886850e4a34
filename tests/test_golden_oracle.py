"""The oracle against the golden fixtures produced by the reference's own backend.

Bit-exact comparisons (np.array_equal): the oracle restates eager-torch rounding exactly.
"""
import numpy as np
import pytest

from oracle import stencil_oracle as O
import oracle
from conftest import Golden, GOLDEN

G = Golden(GOLDEN)
NAMES = sorted(G.cases)


def _formula(name, x, steps, case):
    if name.startswith("mean3_1d"):
        f = O.mean3_1d
    elif name.startswith("jacobi5_2d"):
        f = O.jacobi5_2d
    elif name.startswith("heat7_3d"):
        f = O.heat7_3d
    elif name.startswith("box27_3d"):
        w = case["weights"]
        f = lambda u: O.box27_3d(u, w)  # noqa: E731
    elif name.startswith("star25_3d"):
        from basalto.program import LAPLACIAN8_COEFFS
        f = lambda u: O.star_3d(u, LAPLACIAN8_COEFFS)  # noqa: E731
    else:
        return None
    return O.sweeps(x, f, steps)


@pytest.mark.parametrize("name", NAMES)
def test_formula_oracle_matches_reference(name):
    case = G.cases[name]
    got = _formula(name, G.input(name), case["steps"], case)
    if got is None:
        pytest.skip("reference report stencil: checked through its program")
    ref = G.output(name)
    assert got.dtype == ref.dtype and got.shape == ref.shape
    assert np.array_equal(got, ref)


@pytest.mark.parametrize("name", NAMES)
def test_program_oracle_matches_reference(name):
    case = G.cases[name]
    p = case["program"]
    x = G.input(name)
    f = lambda u: O.eval_program(u, G.terms(name), p["init_zero"], p["boundary"], p["shrink"])  # noqa: E731
    got = O.sweeps(x, f, case["steps"])
    assert np.array_equal(got, G.output(name))


@pytest.mark.parametrize("name", NAMES)
def test_c_oracle_matches_reference(name):
    case = G.cases[name]
    p = case["program"]
    x = G.input(name)
    f = lambda u: oracle.program_c(u, G.terms(name), p["init_zero"], p["boundary"], p["shrink"])  # noqa: E731
    got = O.sweeps(x, f, case["steps"])
    assert np.array_equal(got, G.output(name))


def test_naive_stencil_cpu_restatement_matches_box27():
    """executor.rs:207-289 (float64 box, ascending order, sum from 0) == the 27-point workload."""
    for name in [n for n in NAMES if n.startswith("box27_3d") and G.cases[n]["steps"] == 1]:
        w = G.cases[name]["weights"]
        assert np.array_equal(oracle.naive_box_f64(G.input(name), 1, w), G.output(name))


@pytest.mark.parametrize("name", NAMES)
def test_reference_interceptor_arguments(name):
    """What the reference backend passes to compile_and_execute (compiler.py:77-94)."""
    call = G.cases[name]["reference_call"]
    x = G.input(name)
    assert call["op"] == "stencil"
    assert call["dtype"] == {"float32": "float32", "float64": "float64"}[str(x.dtype)]
    assert call["shape"] == list(x.shape)
    assert call["strides"] == [s // x.itemsize for s in x.strides]
    assert call["device_ptr_z"] == 0


def test_fixture_meta_records_generator():
    assert G.meta["generator"] == "tests/golden/make_golden.py"
    assert len(NAMES) >= 20
