"""The stencil workloads this package is measured on, written as a user writes them.

Each workload is an eager-torch function (what `torch.compile(fn, backend="basalto")`
receives), the equivalent StencilProgram, a seeded input generator and the sweep count.
Inputs generated on the CPU use `torch.Generator().manual_seed(seed)` so CPU and GPU runs
can start from identical grids; the weights of the 27-point box come from
`torch.rand(27, generator=manual_seed(3), dtype=float64) / 27` and its data from a fresh
generator seeded 3.

  mean3_1d    y[i] = (x[i] + x[i+1] + x[i+2]) / 3, fp32 2^24 ~N(0,1) seed 0, valid region
  jacobi5_2d  0.25*(N+S+W+E) fp32 8192^2 ~U(-1,1) seed 1, zero ghosts, 100 sweeps
  heat7_3d    0.4*u + 0.1*(6 neighbours) fp32 512^3 ~U(0,1) seed 2, zero ghosts, 50 steps
  box27_3d    27 weights ~U(0,1/27), fp64 768^3 ~N(0,1) seed 3, zero ghosts, 20 steps
  star25_3d   8th-order Laplacian star r=4, fp32 1024^3 ~N(0,1) seed 4, zero ghosts, 10 steps

`scaling` says how a workload spreads over N GPUs (Z-slabs along axis 0): "strong" splits
the one global grid (heat-7 512^3, star-25 1024^3), "weak" gives every GPU a grid of the
listed size (box-27 768^3 per GPU; the 2-D Jacobi grid), "replicas" runs independent copies
(the 1-D mean, which has no slab axis).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable

import torch
import torch.nn.functional as F

from . import program as P


def mean3_1d(x):
    return (x[..., :-2] + x[..., 1:-1] + x[..., 2:]) / 3.0


def jacobi5_2d(u):
    p = F.pad(u, (1, 1, 1, 1))
    return 0.25 * (p[:-2, 1:-1] + p[2:, 1:-1] + p[1:-1, :-2] + p[1:-1, 2:])


def heat7_3d(u):
    p = F.pad(u, (1, 1, 1, 1, 1, 1))
    c = p[1:-1, 1:-1, 1:-1]
    return 0.4 * c + 0.1 * (p[:-2, 1:-1, 1:-1] + p[2:, 1:-1, 1:-1] + p[1:-1, :-2, 1:-1]
                            + p[1:-1, 2:, 1:-1] + p[1:-1, 1:-1, :-2] + p[1:-1, 1:-1, 2:])


def make_box27_3d(weights) -> Callable:
    """Zero-ghost 27-point box; weights in dz-major, dy, dx order accumulated from zero."""
    w = [float(v) for v in weights]

    def box27_3d(u):
        nz, ny, nx = u.shape
        p = F.pad(u, (1, 1, 1, 1, 1, 1))
        out = torch.zeros_like(u)
        idx = 0
        for dz in range(3):
            for dy in range(3):
                for dx in range(3):
                    out = out + w[idx] * p[dz:dz + nz, dy:dy + ny, dx:dx + nx]
                    idx += 1
        return out

    return box27_3d


def make_star_3d(coeffs=P.LAPLACIAN8_COEFFS) -> Callable:
    """Zero-ghost star of radius len(coeffs)-1: c0*u, then per k the z, y and x pairs."""
    c = [float(v) for v in coeffs]
    R = len(c) - 1

    def star_3d(u):
        nz, ny, nx = u.shape
        p = F.pad(u, (R,) * 6)
        out = c[0] * p[R:R + nz, R:R + ny, R:R + nx]
        for k in range(1, R + 1):
            out = out + c[k] * (p[R + k:R + k + nz, R:R + ny, R:R + nx] + p[R - k:R - k + nz, R:R + ny, R:R + nx])
            out = out + c[k] * (p[R:R + nz, R + k:R + k + ny, R:R + nx] + p[R:R + nz, R - k:R - k + ny, R:R + nx])
            out = out + c[k] * (p[R:R + nz, R:R + ny, R + k:R + k + nx] + p[R:R + nz, R:R + ny, R - k:R - k + nx])
        return out

    return star_3d


def box27_weights(seed: int = 3) -> list[float]:
    g = torch.Generator().manual_seed(seed)
    return (torch.rand(27, generator=g, dtype=torch.float64) / 27).tolist()


def gen_input(kind: str, shape, dtype, seed: int, device="cpu") -> torch.Tensor:
    """Seeded grid: kind in {"randn", "rand", "rand_pm1"}.  CPU generation is the reference
    stream; a CUDA generator with the same seed gives a different (still seeded) grid."""
    dev = torch.device(device)
    g = torch.Generator(device=dev).manual_seed(seed)
    if kind == "randn":
        return torch.randn(shape, generator=g, dtype=dtype, device=dev)
    if kind == "rand":
        return torch.rand(shape, generator=g, dtype=dtype, device=dev)
    if kind == "rand_pm1":
        return torch.rand(shape, generator=g, dtype=dtype, device=dev) * 2 - 1
    raise ValueError(kind)


@dataclass(frozen=True)
class Workload:
    name: str
    fn: Callable
    program: P.StencilProgram
    shape: tuple[int, ...]
    dtype: torch.dtype
    dist: str
    seed: int
    steps: int
    scaling: str = "strong"   # "strong" | "weak" | "replicas" across GPUs

    def global_shape(self, nranks: int = 1) -> tuple[int, ...]:
        """The grid all ranks together hold: the listed grid (strong, replicas) or nranks
        of them stacked along axis 0 (weak)."""
        if self.scaling == "weak" and nranks > 1:
            return (self.shape[0] * nranks,) + tuple(self.shape[1:])
        return tuple(self.shape)

    def label(self) -> str:
        """One name for the configuration, the same in every measurement that runs it."""
        dt = "fp32" if self.dtype == torch.float32 else "fp64"
        per = " per GPU" if self.scaling == "weak" else ""
        return (f"{self.name} {'x'.join(map(str, self.shape))}{per} {dt} {self.dist} seed {self.seed}, "
                f"{self.steps} sweep{'s' if self.steps != 1 else ''} per step"
                f"{' from the unchanged seeded grid' if self.program.boundary == 'zero' else ''}")

    @property
    def points(self) -> int:
        n = 1
        for s in self.shape:
            n *= s
        return n

    @property
    def out_points(self) -> int:
        n = 1
        for s in self.program.out_shape(self.shape):
            n *= s
        return n

    @property
    def elem_size(self) -> int:
        return torch.empty((), dtype=self.dtype).element_size()

    def make_input(self, shape=None, device="cpu") -> torch.Tensor:
        return gen_input(self.dist, tuple(shape or self.shape), self.dtype, self.seed, device)


def _workloads() -> dict[str, Workload]:
    w27 = box27_weights(3)
    return {
        "mean3_1d": Workload("mean3_1d", mean3_1d, P.mean3_1d(), (1 << 24,), torch.float32, "randn", 0, 1,
                             "replicas"),
        "jacobi5_2d": Workload("jacobi5_2d", jacobi5_2d, P.jacobi5_2d(), (8192, 8192), torch.float32,
                               "rand_pm1", 1, 100, "weak"),
        "heat7_3d": Workload("heat7_3d", heat7_3d, P.heat7_3d(), (512, 512, 512), torch.float32, "rand", 2, 50,
                             "strong"),
        "box27_3d": Workload("box27_3d", make_box27_3d(w27), P.box(3, 1, w27), (768, 768, 768), torch.float64,
                             "randn", 3, 20, "weak"),
        "star25_3d": Workload("star25_3d", make_star_3d(), P.star_3d(P.LAPLACIAN8_COEFFS), (1024, 1024, 1024),
                              torch.float32, "randn", 4, 10, "strong"),
    }


WORKLOADS = _workloads()
