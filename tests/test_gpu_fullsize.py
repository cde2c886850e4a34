"""Full-size workloads on the GPU, checked exactly at sampled points.

The grids of the measured configurations (8192^2, 512^3, 768^3 fp64, 1024^3, 2^24) are too
large for the CPU oracle to recompute whole, but every output point depends only on its
neighbourhood: for a sample of points (all corners and faces, plus random interior points)
the input neighbourhood is gathered (exact copies), the oracle folds it in program order,
and the kernel's value must match bit for bit.  These sizes make the march kernel run long
multi-group items, chunk boundaries and full TMA rings, which small grids never reach.
"""
import numpy as np
import pytest
import torch

from oracle import stencil_oracle as O
from conftest import oracle_terms

pytestmark = pytest.mark.gpu


def _sample_points(shape, n, gen):
    pts = [torch.randint(0, s, (n,), generator=gen) for s in shape]
    pts = torch.stack(pts, 1)
    # corners and the middle of every face (boundary handling)
    extra = []
    for c in range(2 ** len(shape)):
        extra.append([(s - 1) if (c >> a) & 1 else 0 for a, s in enumerate(shape)])
    for a, s in enumerate(shape):
        for v in (0, 1, s - 2, s - 1):
            extra.append([v if b == a else shape[b] // 2 for b in range(len(shape))])
    return torch.cat([pts, torch.tensor(extra, dtype=torch.long).clamp(min=0)], 0)


def _gather(x, pts, offsets, boundary):
    vals = []
    for o in offsets:
        idx = pts + torch.tensor(o, dtype=torch.long)
        ok = torch.ones(len(pts), dtype=torch.bool)
        for a, s in enumerate(x.shape):
            ok &= (idx[:, a] >= 0) & (idx[:, a] < s)
        if boundary == "valid":
            assert bool(ok.all())
        safe = torch.where(ok[:, None], idx, torch.zeros_like(idx)).to(x.device)
        v = x[tuple(safe[:, a] for a in range(x.dim()))].cpu().numpy()
        v[~ok.numpy()] = 0
        vals.append(v)
    return vals


def _check(prog, prev, out, gen, n=20000):
    shape = tuple(out.shape)
    pts = _sample_points(shape, n, gen)
    offsets = [o for t in prog.terms for o in t.taps]
    vals = _gather(prev, pts, offsets, prog.boundary)
    dt = np.float32 if prev.dtype == torch.float32 else np.float64
    ref = O.fold_values(vals, oracle_terms(prog), prog.init_zero, dt)
    got = out[tuple(pts[:, a].to(out.device) for a in range(out.dim()))].cpu().numpy()
    assert np.array_equal(got, ref)


@pytest.mark.parametrize("name", ["jacobi5_2d", "heat7_3d", "box27_3d", "star25_3d", "mean3_1d"])
def test_full_size_workload_sampled_exact(name):
    import basalto
    from basalto.workloads import WORKLOADS
    w = WORKLOADS[name]
    prog = w.program
    gen = torch.Generator().manual_seed(7)
    x = w.make_input(device="cuda")
    if prog.boundary == "zero":
        b = torch.empty_like(x)
        prev = basalto.sweeps(prog, x, b, 2)          # two full sweeps first
        prev = prev.clone()
        out = basalto.apply(prog, prev)
    else:
        prev = x
        out = basalto.apply(prog, prev)
    torch.cuda.synchronize()
    assert bool(torch.isfinite(out).all())
    _check(prog, prev, out, gen)
    del x, prev, out
    torch.cuda.empty_cache()
