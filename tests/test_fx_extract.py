"""FX stencil extraction (CPU): recovered programs reproduce eager torch bit for bit, and
graphs that are not linear stencils are refused."""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

from basalto import fx_extract as FX
from basalto import workloads as W
from oracle import stencil_oracle as O
from conftest import oracle_terms


def _capture(fn, *args):
    graphs = []

    def spy(gm, ex):
        graphs.append((gm, list(ex)))
        return gm

    torch._dynamo.reset()
    torch.compile(fn, backend=spy)(*args)
    return graphs[-1]


def _check(fn, x):
    gm, ex = _capture(fn, x)
    prog, tin = FX.extract(gm, ex)
    got = O.eval_program(x.numpy(), oracle_terms(prog), prog.init_zero, prog.boundary, prog.shrink)
    ref = fn(x).numpy()
    assert got.shape == ref.shape
    assert np.array_equal(got, ref)
    return prog


@pytest.mark.parametrize("name", list(W.WORKLOADS))
def test_workload_programs(name):
    w = W.WORKLOADS[name]
    x = w.make_input(tuple(min(s, 12) for s in w.shape))
    gm, ex = _capture(w.fn, x)
    prog, _ = FX.extract(gm, ex)
    assert prog == w.program
    _check(w.fn, x)


def _rollbox(x):  # roll-and-accumulate over a zero-padded copy, as benchmark scripts write it
    r = 1
    out = torch.zeros_like(x)
    p = F.pad(x, (r, r, r, r))
    k = 0
    for dy in range(-r, r + 1):
        for dx in range(-r, r + 1):
            s = torch.roll(p, shifts=(dy, dx), dims=(0, 1))
            out += (0.05 + 0.01 * k) * s[r:r + x.shape[0], r:r + x.shape[1]]
            k += 1
    return out


SPELLINGS = [
    ("scalar_right", lambda u: (u[:-2] + u[2:]) * 0.5, (40,)),
    ("div_sum", lambda u: (u[:, :-2] + u[:, 1:-1] + u[:, 2:]) / 7.0, (9, 30)),
    ("sub_and_neg", lambda u: u[1:-1] - u[:-2] - u[2:], (50,)),
    ("right_nested", lambda u: u[1:-1] + (u[:-2] + u[2:]), (50,)),
    ("neg_term", lambda u: -u[1:-1, 1:-1] + 0.25 * (u[:-2, 1:-1] + u[2:, 1:-1]), (8, 9)),
    ("clone_pad", lambda u: 0.5 * F.pad(u, (1, 1)).clone()[:, :-2] + 0.5 * F.pad(u, (1, 1))[:, 2:], (6, 20)),
    ("roll_box_2d", _rollbox, (11, 14)),
    ("ellipsis", lambda u: u[..., 1:] + u[..., :-1], (5, 6, 7)),
    ("asym_pad", lambda u: 2.0 * F.pad(u, (2, 0))[..., :-2] + F.pad(u, (0, 3))[..., 3:], (30,)),
    ("method_calls", lambda u: u[1:].mul(0.5).add(u[:-1].mul(0.25)), (33,)),
]


@pytest.mark.parametrize("name,fn,shape", SPELLINGS, ids=[s[0] for s in SPELLINGS])
@pytest.mark.parametrize("dtype", [torch.float32, torch.float64])
def test_spellings_reproduce_eager(name, fn, shape, dtype):
    x = torch.randn(shape, dtype=dtype, generator=torch.Generator().manual_seed(3))
    _check(fn, x)


REFUSED = [
    ("matmul", lambda u: u @ u, (4, 4)),
    ("square", lambda u: u * u, (5,)),
    ("affine", lambda u: u[1:] + 1.0, (5,)),
    ("int_index", lambda u: u[1] + u[2], (5, 5)),
    ("strided", lambda u: u[::2] + u[1::2], (8,)),
    ("pad_inside", lambda u: F.pad(u[1:-1], (1, 1)) + u, (8,)),
    ("nested_scale", lambda u: 0.5 * (0.5 * u[1:] + u[:-1]), (8,)),
    ("reflect_pad", lambda u: F.pad(u[None], (1, 1), mode="reflect")[0][:-2] + u, (8,)),
    ("reduction", lambda u: u.sum() * u, (8,)),
    ("roll_wraps", lambda u: torch.roll(u, 1) + u, (8,)),
]


@pytest.mark.parametrize("name,fn,shape", REFUSED, ids=[s[0] for s in REFUSED])
def test_non_stencils_are_refused(name, fn, shape):
    x = torch.randn(shape)
    gm, ex = _capture(fn, x)
    with pytest.raises(FX.Unsupported):
        FX.extract(gm, ex)


def test_two_tensor_inputs_refused():
    gm, ex = _capture(lambda a, b: a[1:] + b[:-1], torch.randn(6), torch.randn(6))
    with pytest.raises(FX.Unsupported):
        FX.extract(gm, ex)
