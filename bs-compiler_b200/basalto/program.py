"""Stencil programs: the exact-order description every kernel of this package executes.

A program is a left fold of terms; each term is an optional scale applied (by multiply or
divide) to a left-to-right sum of taps (shifted reads of the input grid):

    out(p) = ((t0 + t1) + t2) + ...            (init_zero: (((0 + t0) + t1) + ...))
    t_g    = scale_g * (x(p+o1) + x(p+o2) + ...)    or  (...) / scale_g   or  (...)

Every operation is rounded separately in the element type, so a program that lists the
operations of an eager-torch expression in the same order reproduces it bit for bit.

Boundary:
  "zero"  — output shape == input shape, reads outside the grid are 0 (Dirichlet-0 ghost
            cells; the reference's zero padding, crates/basalto-core/src/ir/common.rs:49-63).
  "valid" — taps are relative to the output index and stay inside the input; the output
            shrinks by `shrink[axis]` along each axis (slice-style stencils such as
            `(x[:-2] + x[1:-1] + x[2:]) / 3`).
"""
from __future__ import annotations

import ctypes
import dataclasses
from dataclasses import dataclass, field
from typing import Sequence

from . import _abi

OPS = {"sum": _abi.TERM_SUM, "mul": _abi.TERM_MUL, "div": _abi.TERM_DIV}


@dataclass(frozen=True)
class Term:
    op: str                                # "sum" | "mul" | "div"
    scale: float                           # ignored for "sum"
    taps: tuple[tuple[int, ...], ...]      # offsets in shape order


@dataclass(frozen=True)
class StencilProgram:
    ndim: int
    terms: tuple[Term, ...]
    init_zero: bool = False
    boundary: str = "zero"                 # "zero" | "valid"
    shrink: tuple[int, ...] = field(default=())   # valid only: output = input - shrink
    # Fold every multiplied term after the first as one fused multiply-add,
    # acc = fma(scale, sum, acc) (C-ABI flag BST_PROGRAM_CONTRACT): the reference GPU
    # kernel's `acc += x * c` as LLVM's NVPTX backend contracts it.  Off: bit-identical to
    # eager torch.
    contract: bool = False

    def __post_init__(self):
        if self.ndim not in (1, 2, 3):
            raise ValueError("stencil programs are 1-, 2- or 3-dimensional")
        if not self.terms:
            raise ValueError("a program needs at least one term")
        for t in self.terms:
            if t.op not in OPS:
                raise ValueError(f"unknown term op {t.op!r}")
            if not t.taps:
                raise ValueError("every term needs at least one tap")
            for o in t.taps:
                if len(o) != self.ndim:
                    raise ValueError("tap offsets must have ndim entries")
        if self.boundary not in ("zero", "valid"):
            raise ValueError("boundary is 'zero' or 'valid'")
        if self.boundary == "valid" and len(self.shrink) != self.ndim:
            raise ValueError("a valid-region program needs one shrink value per axis")

    @property
    def ntaps(self) -> int:
        return sum(len(t.taps) for t in self.terms)

    def radius(self) -> tuple[int, ...]:
        """Per-axis reach of the taps around the output point (zero boundary)."""
        r = [0] * self.ndim
        for t in self.terms:
            for o in t.taps:
                for a, v in enumerate(o):
                    r[a] = max(r[a], abs(v))
        return tuple(r)

    def out_shape(self, shape: Sequence[int]) -> tuple[int, ...]:
        if len(shape) != self.ndim:
            raise ValueError(f"program is {self.ndim}-D, grid has shape {tuple(shape)}")
        if self.boundary == "zero":
            return tuple(int(s) for s in shape)
        return tuple(int(s) - int(k) for s, k in zip(shape, self.shrink))

    def to_c(self, shape: Sequence[int] | None = None) -> _abi.CProgram:
        if self.ntaps > _abi.MAX_TAPS or len(self.terms) > _abi.MAX_TERMS:
            raise ValueError("program exceeds the C ABI limits")
        p = _abi.CProgram()
        p.ndim = self.ndim
        p.ntaps = self.ntaps
        p.nterms = len(self.terms)
        p.init_zero = 1 if self.init_zero else 0
        p.boundary = _abi.BOUNDARY_ZERO if self.boundary == "zero" else _abi.BOUNDARY_VALID
        p.flags = _abi.BST_PROGRAM_CONTRACT if self.contract else 0
        if self.boundary == "valid":
            if shape is None:
                raise ValueError("a valid-region program needs the input shape")
            for a, v in enumerate(self.out_shape(shape)):
                p.out_shape[a] = v
        k = 0
        for g, t in enumerate(self.terms):
            p.term_first[g] = k
            p.term_count[g] = len(t.taps)
            p.term_op[g] = OPS[t.op]
            p.term_scale[g] = float(t.scale)
            for o in t.taps:
                for a, v in enumerate(o):
                    p.tap[k][a] = int(v)
                k += 1
        return p

    def contracted(self, on: bool = True) -> "StencilProgram":
        """This program with fused multiply-add folding switched on (or off)."""
        return dataclasses.replace(self, contract=bool(on))

    def pack(self, shape: Sequence[int] | None = None) -> bytes:
        """The program as the raw bytes of a C `bst_program` (for the interceptor)."""
        return bytes(self.to_c(shape))


# ---- programs of the workloads and of the reference's operator ------------------------

def box(ndim: int, radius: int, coeffs: Sequence[float] | None = None, descending: bool = False) -> StencilProgram:
    """Zero-padded (2r+1)^ndim box accumulated from 0, one weighted term per tap.

    Ascending offsets, slowest axis major, with isotropic weights 1/(2r+1)^ndim unless
    `coeffs` is given: the reference's stencil operator (crates/basalto-core/src/
    flir_builder.rs:58-65, crates/basalto-tree/src/executor.rs:207-289).  `descending`
    gives the reverse tap order, as a roll-and-accumulate loop over ascending shifts
    produces (report/scripts/stencil_benchmark.py:14-58 rolls by +d and so reads x[i-d]).
    """
    w = 2 * radius + 1
    n = w ** ndim
    if coeffs is not None and len(coeffs) != n:
        raise ValueError(f"expected {n} coefficients")
    offs = []
    for k in range(n):
        o, r = [], k
        for _ in range(ndim):
            o.append(r % w - radius)
            r //= w
        offs.append(tuple(reversed(o)))
    iso = 1.0 / n
    terms = [Term("mul", float(coeffs[k]) if coeffs is not None else iso, (offs[k],)) for k in range(n)]
    if descending:
        terms = [Term(t.op, t.scale, (tuple(-v for v in t.taps[0]),)) for t in terms]
    return StencilProgram(ndim, tuple(terms), init_zero=True)


def mean3_1d(divisor: float = 3.0) -> StencilProgram:
    """(x[i] + x[i+1] + x[i+2]) / divisor over the valid region (output length n-2)."""
    return StencilProgram(1, (Term("div", divisor, ((0,), (1,), (2,))),), boundary="valid", shrink=(2,))


def jacobi5_2d(scale: float = 0.25) -> StencilProgram:
    """scale * (u[y-1] + u[y+1] + u[x-1] + u[x+1]) with zero ghost cells."""
    return StencilProgram(2, (Term("mul", scale, ((-1, 0), (1, 0), (0, -1), (0, 1))),))


def heat7_3d(c0: float = 0.4, c1: float = 0.1) -> StencilProgram:
    """c0 * u + c1 * (u[z-1] + u[z+1] + u[y-1] + u[y+1] + u[x-1] + u[x+1]), zero ghosts."""
    nb = ((-1, 0, 0), (1, 0, 0), (0, -1, 0), (0, 1, 0), (0, 0, -1), (0, 0, 1))
    return StencilProgram(3, (Term("mul", c0, ((0, 0, 0),)), Term("mul", c1, nb)))


def star_3d(coeffs: Sequence[float]) -> StencilProgram:
    """c0 * u + sum_{k=1..R} [c_k (u[z+k] + u[z-k]) + c_k (u[y+k] + u[y-k]) + c_k (u[x+k] + u[x-k])]."""
    R = len(coeffs) - 1
    terms = [Term("mul", float(coeffs[0]), ((0, 0, 0),))]
    for k in range(1, R + 1):
        for ax in range(3):
            p = [0, 0, 0]
            m = [0, 0, 0]
            p[ax], m[ax] = k, -k
            terms.append(Term("mul", float(coeffs[k]), (tuple(p), tuple(m))))
    return StencilProgram(3, tuple(terms))


# 8th-order central second derivative (1/h^2 = 1): centre -205/72, then 8/5, -1/5, 8/315, -1/560;
# the 3-D Laplacian has centre 3 * (-205/72).
LAPLACIAN8_COEFFS = (3.0 * (-205.0 / 72.0), 8.0 / 5.0, -1.0 / 5.0, 8.0 / 315.0, -1.0 / 560.0)
