"""Recover a StencilProgram from the FX graph Dynamo hands the backend.

The reference backend only substring-matches FX targets to pick "stencil" and always runs
the isotropic box of the op's radius (python/basalto/compiler.py:10-40,
crates/basalto-core/src/flir_builder.rs:58-65).  Here the graph itself is interpreted
symbolically: every tensor value is either a *view* of the single input grid (a shifted
window, possibly zero-padded or rolled) or an expression over such views.  A graph whose
output is a left fold of (scale *|/ sum-of-views) terms becomes a program with the same
operation order, so the kernels reproduce eager torch bit for bit.  Anything else raises
Unsupported and the backend leaves the graph to eager execution.

Recognised: slicing (`x[a:b]`, `...`), F.pad (constant zero), torch.roll, +, +=, -, unary -,
* and / by Python scalars, torch.zeros_like as the accumulator seed, clone/contiguous.
"""
from __future__ import annotations

import math
import operator
from dataclasses import dataclass

import torch
import torch.fx

from .program import StencilProgram, Term


class Unsupported(Exception):
    """The graph is not a single-input linear stencil this package can run."""


INF = 1 << 60


@dataclass(frozen=True)
class AxisView:
    off: int      # view index i reads input index i + off
    n: int        # view extent
    zlo: int      # reads must stay in [zlo, zhi); outside [0, N) they read 0 (zero pads)
    zhi: int
    wlo: int      # view indices valid without wrap-around (torch.roll)
    whi: int


@dataclass(frozen=True)
class Leaf:
    axes: tuple[AxisView, ...]

    @property
    def shape(self):
        return tuple(a.n for a in self.axes)


@dataclass(frozen=True)
class Zero:
    shape: tuple[int, ...]


@dataclass(frozen=True)
class Add:
    a: object
    b: object
    shape: tuple[int, ...]


@dataclass(frozen=True)
class Scale:
    e: object
    s: float
    op: str        # "mul" | "div"
    shape: tuple[int, ...]


def _shape(v):
    return v.shape


_ADD = {operator.add, operator.iadd, torch.add}
_SUB = {operator.sub, operator.isub, torch.sub}
_MUL = {operator.mul, operator.imul, torch.mul}
_DIV = {operator.truediv, operator.itruediv, torch.div, torch.true_divide}
_NEG = {operator.neg, torch.neg}
_PAD = {torch.nn.functional.pad}
try:  # the builtin Dynamo records for F.pad
    _PAD.add(torch._C._nn.pad)
except AttributeError:  # pragma: no cover
    pass
_ROLL = {torch.roll}
_ZEROS_LIKE = {torch.zeros_like}
_METHODS_IDENTITY = {"clone", "contiguous"}


def _is_num(v):
    return isinstance(v, (int, float)) and not isinstance(v, bool)


def _is_tensor_expr(v):
    return isinstance(v, (Leaf, Zero, Add, Scale))


class _Interp:
    def __init__(self, in_shape):
        self.in_shape = tuple(int(s) for s in in_shape)

    # -- views ---------------------------------------------------------------------
    def input_leaf(self):
        return Leaf(tuple(AxisView(0, n, 0, n, -INF, INF) for n in self.in_shape))

    def slice_(self, v, idx):
        if not isinstance(v, Leaf):
            raise Unsupported("slicing is only supported on views of the input")
        if not isinstance(idx, tuple):
            idx = (idx,)
        nd = len(v.axes)
        if sum(1 for i in idx if i is Ellipsis) > 1:
            raise Unsupported("more than one Ellipsis")
        if Ellipsis in idx:
            k = idx.index(Ellipsis)
            fill = nd - (len(idx) - 1)
            idx = idx[:k] + (slice(None),) * fill + idx[k + 1:]
        if len(idx) > nd:
            raise Unsupported("too many indices")
        idx = idx + (slice(None),) * (nd - len(idx))
        axes = []
        for ax, s in zip(v.axes, idx):
            if not isinstance(s, slice):
                raise Unsupported("only slices are supported (no integer or tensor indexing)")
            if s.step not in (None, 1):
                raise Unsupported("strided slices are not stencils")
            a, b, _ = s.indices(ax.n)
            b = max(a, b)
            axes.append(AxisView(ax.off + a, b - a, ax.zlo, ax.zhi, ax.wlo - a, ax.whi - a))
        return Leaf(tuple(axes))

    def pad(self, v, pads, mode="constant", value=None):
        if not isinstance(v, Leaf):
            raise Unsupported("padding is only supported on views of the input")
        if mode != "constant" or (value not in (None, 0, 0.0)):
            raise Unsupported("only constant zero padding")
        pads = list(pads)
        if len(pads) % 2 or len(pads) // 2 > len(v.axes):
            raise Unsupported("bad pad spec")
        axes = list(v.axes)
        nd = len(axes)
        for k in range(len(pads) // 2):
            a = nd - 1 - k
            lo, hi = int(pads[2 * k]), int(pads[2 * k + 1])
            ax = axes[a]
            N = self.in_shape[a]
            if lo < 0 or hi < 0:
                raise Unsupported("negative padding")
            if ax.wlo > 0 or ax.whi < ax.n:
                raise Unsupported("padding a rolled view")
            # Zeros land next to the view window; they match zero ghost cells only when the
            # window reaches the grid edge on that side.
            if lo and ax.off != 0:
                raise Unsupported("zero padding inside the grid")
            if hi and ax.off + ax.n != N:
                raise Unsupported("zero padding inside the grid")
            axes[a] = AxisView(ax.off - lo, ax.n + lo + hi, ax.zlo - lo, ax.zhi + hi, -INF, INF)
        return Leaf(tuple(axes))

    def roll(self, v, shifts, dims):
        if not isinstance(v, Leaf):
            raise Unsupported("roll is only supported on views of the input")
        if dims is None:
            raise Unsupported("roll over the flattened tensor")
        if isinstance(shifts, int):
            shifts = (shifts,)
        if isinstance(dims, int):
            dims = (dims,)
        if len(shifts) != len(dims):
            raise Unsupported("roll shifts/dims mismatch")
        axes = list(v.axes)
        for s, d in zip(shifts, dims):
            d = d % len(axes)
            ax = axes[d]
            s = int(s)
            # rolled[i] = view[i - s] while 0 <= i - s < n (wrap-around is not a stencil)
            lo = max(0, ax.wlo) + s
            hi = min(ax.n, ax.whi) + s
            axes[d] = AxisView(ax.off - s, ax.n, ax.zlo, ax.zhi, lo, hi)
        return Leaf(tuple(axes))

    # -- arithmetic ---------------------------------------------------------------------
    def add(self, a, b):
        if not (_is_tensor_expr(a) and _is_tensor_expr(b)):
            raise Unsupported("adding a scalar is not a linear stencil")
        if _shape(a) != _shape(b):
            raise Unsupported("broadcasting add")
        return Add(a, b, _shape(a))

    def scale(self, e, s, op):
        if not _is_tensor_expr(e):
            raise Unsupported("scale of a non-tensor")
        if not math.isfinite(float(s)):
            raise Unsupported("non-finite scale")
        return Scale(e, float(s), op, _shape(e))


def _eval_graph(gm: torch.fx.GraphModule, args):
    """Symbolically run `gm` on (tensor, ints...) args; returns (expr, input_index, in_shape)."""
    placeholders = [n for n in gm.graph.nodes if n.op == "placeholder"]
    if len(placeholders) != len(args):
        raise Unsupported("argument count mismatch")
    tensors = [i for i, a in enumerate(args) if isinstance(a, torch.Tensor)]
    if len(tensors) != 1:
        raise Unsupported("a stencil graph has exactly one tensor input")
    tin = tensors[0]
    x = args[tin]
    if x.dim() < 1 or x.dim() > 3:
        raise Unsupported("only 1-D, 2-D and 3-D grids")
    it = _Interp(x.shape)
    env = {}
    out = None
    for node in gm.graph.nodes:
        if node.op == "placeholder":
            k = placeholders.index(node)
            a = args[k]
            env[node] = it.input_leaf() if k == tin else (int(a) if isinstance(a, (int, torch.SymInt)) else a)
            continue
        if node.op == "output":
            res = node.args[0]
            if isinstance(res, (tuple, list)):
                if len(res) != 1:
                    raise Unsupported("a stencil graph has exactly one output")
                res = res[0]
            out = env[res] if isinstance(res, torch.fx.Node) else res
            break
        a = torch.fx.node.map_arg(node.args, lambda n: env[n])
        kw = torch.fx.node.map_arg(node.kwargs, lambda n: env[n])
        if node.op == "call_function":
            env[node] = _call_function(it, node.target, a, kw)
        elif node.op == "call_method":
            env[node] = _call_method(it, node.target, a, kw)
        else:
            raise Unsupported(f"node kind {node.op}")
    if not _is_tensor_expr(out):
        raise Unsupported("output is not a tensor expression")
    return out, tin, tuple(int(s) for s in x.shape)


def _call_function(it, t, a, kw):
    if t is operator.getitem:
        v, idx = a
        if isinstance(v, (tuple, list, torch.Size)):
            return v[idx]
        return it.slice_(v, idx)
    if t is getattr:
        v, name = a
        if name == "shape" and isinstance(v, Leaf):
            return v.shape
        raise Unsupported(f"getattr {name}")
    if t in _ADD:
        if kw.get("alpha", 1) != 1:
            raise Unsupported("add with alpha")
        if all(_is_num(v) for v in a):
            return a[0] + a[1]
        return it.add(a[0], a[1])
    if t in _SUB:
        if kw.get("alpha", 1) != 1:
            raise Unsupported("sub with alpha")
        if all(_is_num(v) for v in a):
            return a[0] - a[1]
        # u - v == u + (-1 * v) exactly in IEEE arithmetic
        return it.add(a[0], it.scale(a[1], -1.0, "mul"))
    if t in _MUL:
        u, v = a
        if _is_num(u) and _is_num(v):
            return u * v
        if _is_num(u):
            return it.scale(v, u, "mul")
        if _is_num(v):
            return it.scale(u, v, "mul")
        raise Unsupported("tensor * tensor")
    if t in _DIV:
        if kw.get("rounding_mode") is not None:
            raise Unsupported("rounded division")
        u, v = a
        if _is_num(u) and _is_num(v):
            return u / v
        if _is_num(v):
            return it.scale(u, v, "div")
        raise Unsupported("division by a tensor")
    if t in _NEG:
        return it.scale(a[0], -1.0, "mul")
    if t in _ZEROS_LIKE:
        if set(kw) - {"dtype", "layout", "device", "pin_memory", "memory_format"} or kw.get("dtype") is not None:
            raise Unsupported("zeros_like with a dtype change")
        return Zero(_shape(a[0]))
    if t in _PAD:
        v = a[0]
        pads = a[1] if len(a) > 1 else kw["pad"]
        mode = a[2] if len(a) > 2 else kw.get("mode", "constant")
        value = a[3] if len(a) > 3 else kw.get("value", None)
        return it.pad(v, pads, mode, value)
    if t in _ROLL:
        shifts = a[1] if len(a) > 1 else kw["shifts"]
        dims = a[2] if len(a) > 2 else kw.get("dims")
        return it.roll(a[0], shifts, dims)
    raise Unsupported(f"call_function {getattr(t, '__name__', t)}")


def _call_method(it, name, a, kw):
    self = a[0]
    if name in _METHODS_IDENTITY:
        return self
    if name == "size":
        s = self.shape
        return s[a[1]] if len(a) > 1 else s
    if name in ("add", "add_", "__add__", "__iadd__"):
        return _call_function(it, operator.add, a, kw)
    if name in ("sub", "sub_"):
        return _call_function(it, operator.sub, a, kw)
    if name in ("mul", "mul_", "__mul__", "__rmul__"):
        return _call_function(it, operator.mul, a, kw)
    if name in ("div", "div_", "true_divide"):
        return _call_function(it, operator.truediv, a, kw)
    if name in ("neg",):
        return _call_function(it, operator.neg, a, kw)
    if name == "roll":
        return _call_function(it, torch.roll, a, kw)
    raise Unsupported(f"call_method {name}")


def _left_spine(e):
    items = []
    while isinstance(e, Add):
        items.append(e.b)
        e = e.a
    items.append(e)
    return items[::-1]


def _leaf_sum(e):
    items = _left_spine(e)
    if not all(isinstance(i, Leaf) for i in items):
        raise Unsupported("a term must be a left-to-right sum of grid views")
    return items


def to_program(expr, in_shape) -> StencilProgram:
    """Turn an interpreted output expression into a StencilProgram (or raise Unsupported)."""
    items = _left_spine(expr)
    init_zero = False
    if isinstance(items[0], Zero):
        init_zero = True
        items = items[1:]
    if not items:
        raise Unsupported("the graph computes a constant")
    out_shape = tuple(expr.shape)
    nd = len(in_shape)
    terms = []
    leaves = []
    for it in items:
        if isinstance(it, Zero):
            raise Unsupported("zero tensor inside the fold")
        if isinstance(it, Scale):
            inner = _leaf_sum(it.e)
            terms.append((it.op, it.s, inner))
        else:
            terms.append(("sum", 1.0, _leaf_sum(it)))
        leaves.extend(terms[-1][2])
    for lf in leaves:
        if lf.shape != out_shape:
            raise Unsupported("views of different shapes")
        for a, ax in enumerate(lf.axes):
            if ax.wlo > 0 or ax.whi < ax.n:
                raise Unsupported("a roll wraps around")
            if ax.off < ax.zlo or ax.off + ax.n > ax.zhi:
                raise Unsupported("a view reads beyond its padding")
    same = out_shape == tuple(in_shape)
    if same:
        boundary, shrink = "zero", ()
    else:
        for lf in leaves:
            for a, ax in enumerate(lf.axes):
                if ax.off < 0 or ax.off + ax.n > in_shape[a]:
                    raise Unsupported("a shrinking stencil that also reads zero padding")
        boundary, shrink = "valid", tuple(in_shape[a] - out_shape[a] for a in range(nd))
    tl = tuple(Term(op, s, tuple(tuple(ax.off for ax in lf.axes) for lf in lv)) for op, s, lv in terms)
    return StencilProgram(nd, tl, init_zero=init_zero, boundary=boundary, shrink=shrink)


def extract(gm: torch.fx.GraphModule, args):
    """Returns (program, tensor_arg_index) for a stencil graph; raises Unsupported otherwise."""
    expr, tin, in_shape = _eval_graph(gm, args)
    x = args[tin]
    if x.dtype not in (torch.float32, torch.float64):
        raise Unsupported(f"dtype {x.dtype}")
    return to_program(expr, in_shape), tin
