"""GPU parity of fused multiply-add programs (BST_PROGRAM_CONTRACT), bit for bit.

With the flag, every multiplied term after the first folds as one fma — the arithmetic of
the reference's own GPU kernel once LLVM's NVPTX backend contracts its `acc += x * c`.  The
kernels must equal the C oracle's fma()/fmaf() fold exactly, on the TMA catalog kernels
(3-D heat, 27-point boxes in both tap orders, the r=4 star, the weighted 7-point star), the
direct kernels (strided views) and the runtime-table kernel (2-D / 1-D boxes), single sweeps
and multi-sweep runs, and through torch.compile with BASALTO_FP_CONTRACT=1.  Against eager
(separately rounded) results the difference is rounding only.
"""
import numpy as np
import pytest
import torch

import oracle
from conftest import oracle_terms

pytestmark = pytest.mark.gpu


def _programs():
    from basalto import program as P
    from basalto import workloads as W
    from basalto.program import StencilProgram, Term
    wstar = StencilProgram(3, tuple(Term("mul", c, (o,)) for c, o in zip(
        (0.3, 0.11, 0.12, 0.13, 0.14, 0.15, 0.16),
        ((0, 0, 0), (-1, 0, 0), (1, 0, 0), (0, -1, 0), (0, 1, 0), (0, 0, -1), (0, 0, 1)))))
    return {
        "heat7_3d": P.heat7_3d(),
        "box27_3d": P.box(3, 1, W.box27_weights()),
        "box27_desc": P.box(3, 1, W.box27_weights(), descending=True),
        "star25_3d": P.star_3d(P.LAPLACIAN8_COEFFS),
        "wstar7_3d": wstar,
        "box2d_r2": P.box(2, 2),
        "box1d_r3": P.box(1, 3),
    }


SHAPES = {1: [(1000,), (4096,), (37,)], 2: [(33, 128), (100, 1000), (7, 13)],
          3: [(17, 33, 64), (9, 40, 128), (33, 17, 100), (4, 5, 6)]}


def _ref(x, prog):
    return oracle.program_c(x, oracle_terms(prog), init_zero=prog.init_zero, contract=True)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float64])
@pytest.mark.parametrize("key", list(_programs()))
def test_contracted_kernels_equal_fma_oracle(key, dtype):
    import basalto
    prog = _programs()[key].contracted()
    g = torch.Generator().manual_seed(21)
    for shape in SHAPES[prog.ndim]:
        x = torch.randn(shape, generator=g, dtype=dtype)
        got = basalto.apply(prog, x.cuda()).cpu().numpy()
        ref = _ref(x.numpy(), prog)
        assert np.array_equal(got, ref), f"{key} {shape} {dtype}"
        plain = basalto.apply(prog.contracted(False), x.cuda()).cpu().numpy()
        tol = 1e-6 if dtype == torch.float32 else 1e-12
        assert np.abs(got - plain).max() <= tol * max(np.abs(plain).max(), 1e-30)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float64])
def test_contracted_strided_views(dtype):
    import basalto
    prog = _programs()["box27_3d"].contracted()
    base = torch.randn(20, 30, 70, dtype=dtype, generator=torch.Generator().manual_seed(4))
    x = base[1:19, 2:29, 3:67]  # a view: the direct kernel
    got = basalto.apply(prog, x.cuda()).cpu().numpy()
    assert np.array_equal(got, _ref(np.ascontiguousarray(x.numpy()), prog))


@pytest.mark.parametrize("dtype", [torch.float32, torch.float64])
def test_contracted_sweeps(dtype):
    import basalto
    for key, shape, n in (("heat7_3d", (20, 24, 64), 4), ("box27_3d", (16, 18, 64), 3), ("star25_3d", (18, 20, 32), 2)):
        prog = _programs()[key].contracted()
        x = torch.randn(shape, dtype=dtype, generator=torch.Generator().manual_seed(6))
        a = x.cuda()
        res = basalto.sweeps(prog, a, torch.empty_like(a), n).cpu().numpy()
        ref = x.numpy()
        for _ in range(n):
            ref = _ref(ref, prog)
        assert np.array_equal(res, ref), key


def test_torch_compile_with_fp_contract(monkeypatch):
    import basalto  # noqa: F401  (registers the backend)
    from basalto import workloads as W
    from basalto import program as P
    monkeypatch.setenv("BASALTO_FP_CONTRACT", "1")
    torch._dynamo.reset()
    fn = torch.compile(W.heat7_3d, backend="basalto")
    x = torch.rand(24, 20, 64, generator=torch.Generator().manual_seed(2))
    got = fn(x.cuda()).cpu().numpy()
    torch._dynamo.reset()
    ref = _ref(x.numpy(), P.heat7_3d().contracted())
    assert np.array_equal(got, ref)
    assert not np.array_equal(got, W.heat7_3d(x).numpy())  # really the fused fold


@pytest.mark.parametrize("name,dtype,sweeps", [("box27", torch.float32, 1), ("box27", torch.float32, 20),
                                               ("box27", torch.float64, 1), ("box27", torch.float64, 20),
                                               ("star25", torch.float32, 1), ("star25", torch.float32, 10)])
def test_fused_mode_error_against_separately_rounded(name, dtype, sweeps):
    """Fused multiply-add mode against the separately rounded result (the reference's
    user-visible arithmetic) on a 160 x 192 x 256 grid, one sweep and a full multi-sweep run.

    Normwise, max|fused - exact| / max|exact| stays within the stated tolerance (1e-6 fp32,
    1e-12 fp64).  Pointwise it does not: where the terms of a point nearly cancel, its value is
    small and one rounding less shifts it by a large fraction of itself (up to ~3e-2 fp32,
    ~6e-11 fp64 measured).  With the denominator floored at 1e-3 x max|exact| the pointwise
    error is bounded by 2e-4 (fp32) and 1e-12 (fp64)."""
    import basalto
    from basalto import program as P
    from basalto import workloads as W
    prog = P.box(3, 1, W.box27_weights()) if name == "box27" else P.star_3d(P.LAPLACIAN8_COEFFS)
    g = torch.Generator(device="cuda").manual_seed(12)
    x = torch.randn((160, 192, 256), generator=g, dtype=dtype, device="cuda")
    a, b = x.clone(), torch.empty_like(x)
    exact = basalto.sweeps(prog, a, b, sweeps).to(torch.float64)
    a2, b2 = x.clone(), torch.empty_like(x)
    fused = basalto.sweeps(prog.contracted(), a2, b2, sweeps).to(torch.float64)
    diff = (fused - exact).abs()
    mag = exact.abs()
    top = float(mag.max())
    normwise = float(diff.max()) / top
    floored = float((diff / torch.clamp(mag, min=1e-3 * top)).max())
    pointwise = float((diff / torch.clamp(mag, min=torch.finfo(torch.float64).tiny)).max())
    tol = 1e-6 if dtype == torch.float32 else 1e-12
    print(f"{name} {dtype} {sweeps} sweeps: normwise {normwise:.2e} pointwise {pointwise:.2e} "
          f"floored(1e-3 max) {floored:.2e}")
    assert normwise <= tol
    assert floored <= (2e-4 if dtype == torch.float32 else 1e-12)
    assert bool(torch.isfinite(fused).all())
