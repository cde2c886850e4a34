"""fp32 division terms of the catalog kernels equal IEEE division bit for bit.

The 1-D mean (x[i] + x[i+1] + x[i+2]) / d runs on the catalog line kernel, whose division term
uses a reciprocal and two quotient corrections (div_by in bst_types.cuh) instead of an IEEE
divide.  Inputs hold one value in every third element and zeros between, so each output is a
single value divided by d; the reference is CUDA's IEEE division of a tensor by a tensor (eager
CUDA torch divides by a Python scalar through its reciprocal, so it is not used).
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _spread(v):
    x = torch.zeros(3 * v.numel(), dtype=torch.float32, device=v.device)
    x[0::3] = v
    return x


def _mismatches(d, v):
    import basalto
    from basalto import program as P
    x = _spread(v)
    n0 = basalto.launch_count()
    y = basalto.apply(P.mean3_1d(d), x)
    assert basalto.launch_count() > n0
    ref = (x[:-2] + x[1:-1] + x[2:]) / torch.full_like(x[:-2], d)
    nan = torch.isnan(ref)
    if not torch.equal(torch.isnan(y), nan):
        return -1
    yb = torch.where(nan, 0, y.view(torch.int32))
    rb = torch.where(nan, 0, ref.view(torch.int32))
    return int((yb != rb).sum().item())


def test_division_by_three_every_fp32_value():
    """All 2^32 bit patterns (zeros, subnormals, infinities and NaNs included) divided by 3."""
    chunk = 1 << 27
    bad = 0
    for c in range(1 << 5):
        lo = -(1 << 31) + c * chunk
        v = torch.arange(lo, lo + chunk, dtype=torch.int32, device="cuda").view(torch.float32)
        m = _mismatches(3.0, v)
        assert m >= 0, "NaN positions differ"
        bad += m
    assert bad == 0


@pytest.mark.parametrize("d", [3.0, 7.0, 0.1, 1 / 3, 1.5, 2.0, -3.0, 65537.0, 1e-18, 1e18, 1e-20, 1e25, 3e-39])
def test_division_by_other_constants(d):
    """Random values over the whole exponent range plus special values, for divisors inside the
    corrected range, powers of two, and divisors outside it (which use IEEE division)."""
    g = np.random.default_rng(int(abs(np.float32(d)).view(np.int32)))
    n = 1 << 22
    bits = g.integers(-(1 << 31), 1 << 31, n, dtype=np.int64).astype(np.int32)
    special = np.array([0.0, -0.0, np.inf, -np.inf, np.nan, 1e-45, -1e-45, 1e-40, 2.0 ** -60, 2.0 ** 60,
                        np.nextafter(np.float32(2.0 ** -60), np.float32(0)),
                        np.nextafter(np.float32(2.0 ** 60), np.float32(np.inf)),
                        3.4028235e38, -3.4028235e38, 1.0, 3.0, 9.0], dtype=np.float32)
    v = np.concatenate([bits.view(np.float32), special])
    assert _mismatches(d, torch.from_numpy(v).cuda()) == 0
