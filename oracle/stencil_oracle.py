"""CPU oracle for the stencil hot path — TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use this module, and
only as the checker; the product path never imports it.

What it restates.  The reference's user-visible result is eager PyTorch: its Dynamo backend
returns the unmodified graph (python/basalto/compiler.py:95), so `torch.compile(f,
backend="basalto")(x)` equals `f(x)` run op by op.  Each eager op rounds separately in the
tensor dtype; a Python scalar is applied in that dtype (`0.4 * t` multiplies by
float32(0.4)) and `t / 3.0` is IEEE division on the CPU.  The functions below restate the
workloads' formulas with numpy in exactly that order, and `eval_program` restates the
generic program semantics (a left fold of scaled tap sums), which also covers the
reference's own CPU check `Executor::naive_stencil_cpu`
(crates/basalto-tree/src/executor.rs:207-289: zero-padded same-size box, coefficient index
slowest-axis-major, `sum = 0; sum += val * coeff`) when evaluated in float64.

Pinned by tests/golden/*.npz, produced by running the reference's own backend
(python/basalto/compiler.py) on seeded inputs (tests/golden/make_golden.py).
"""
from __future__ import annotations

import numpy as np

# ---- the workload formulas ---------------------------------------------------------


def mean3_1d(x: np.ndarray) -> np.ndarray:
    """(x[:-2] + x[1:-1] + x[2:]) / 3.0 — README.md:90-92 of the reference."""
    t = x.dtype.type
    return (x[:-2] + x[1:-1] + x[2:]) / t(3.0)


def jacobi5_2d(u: np.ndarray, scale: float = 0.25) -> np.ndarray:
    """scale * (((u[y-1] + u[y+1]) + u[x-1]) + u[x+1]) with zero ghost cells."""
    t = u.dtype.type
    p = np.pad(u, 1)
    return t(scale) * (((p[:-2, 1:-1] + p[2:, 1:-1]) + p[1:-1, :-2]) + p[1:-1, 2:])


def heat7_3d(u: np.ndarray, c0: float = 0.4, c1: float = 0.1) -> np.ndarray:
    """c0*u + c1*(((((u[z-1]+u[z+1])+u[y-1])+u[y+1])+u[x-1])+u[x+1]), zero ghosts."""
    t = u.dtype.type
    p = np.pad(u, 1)
    c = p[1:-1, 1:-1, 1:-1]
    s = p[:-2, 1:-1, 1:-1] + p[2:, 1:-1, 1:-1]
    s = s + p[1:-1, :-2, 1:-1]
    s = s + p[1:-1, 2:, 1:-1]
    s = s + p[1:-1, 1:-1, :-2]
    s = s + p[1:-1, 1:-1, 2:]
    return t(c0) * c + t(c1) * s


def box27_3d(u: np.ndarray, w) -> np.ndarray:
    """Zero-ghost box, out = 0; out = out + w[k] * u[shift_k] for k in dz, dy, dx order."""
    t = u.dtype.type
    nz, ny, nx = u.shape
    p = np.pad(u, 1)
    out = np.zeros_like(u)
    k = 0
    for dz in range(3):
        for dy in range(3):
            for dx in range(3):
                out = out + t(w[k]) * p[dz:dz + nz, dy:dy + ny, dx:dx + nx]
                k += 1
    return out


def star_3d(u: np.ndarray, c) -> np.ndarray:
    """c0*u, then per k = 1..R: + c_k (z pair), + c_k (y pair), + c_k (x pair); zero ghosts."""
    t = u.dtype.type
    R = len(c) - 1
    nz, ny, nx = u.shape
    p = np.pad(u, R)

    def v(dz, dy, dx):
        return p[R + dz:R + dz + nz, R + dy:R + dy + ny, R + dx:R + dx + nx]

    out = t(c[0]) * v(0, 0, 0)
    for k in range(1, R + 1):
        out = out + t(c[k]) * (v(k, 0, 0) + v(-k, 0, 0))
        out = out + t(c[k]) * (v(0, k, 0) + v(0, -k, 0))
        out = out + t(c[k]) * (v(0, 0, k) + v(0, 0, -k))
    return out


# ---- generic programs ---------------------------------------------------------------
# terms: sequence of (op, scale, taps) with op in {"sum", "mul", "div"} and taps a
# sequence of per-axis offsets (relative to the output index).


def _views(x, terms, boundary, shrink):
    nd = x.ndim
    if boundary == "zero":
        R = [0] * nd
        for _, _, taps in terms:
            for o in taps:
                for a in range(nd):
                    R[a] = max(R[a], abs(o[a]))
        p = np.pad(x, [(r, r) for r in R])
        out_shape = x.shape

        def view(o):
            return p[tuple(slice(R[a] + o[a], R[a] + o[a] + out_shape[a]) for a in range(nd))]
    else:
        out_shape = tuple(x.shape[a] - shrink[a] for a in range(nd))

        def view(o):
            return x[tuple(slice(o[a], o[a] + out_shape[a]) for a in range(nd))]
    return view, out_shape


def eval_program(x: np.ndarray, terms, init_zero=False, boundary="zero", shrink=()) -> np.ndarray:
    t = x.dtype.type
    view, out_shape = _views(x, terms, boundary, shrink)
    acc = None
    for g, (op, scale, taps) in enumerate(terms):
        s = view(taps[0]).copy()
        for o in taps[1:]:
            s = s + view(o)
        if op == "mul":
            s = t(scale) * s
        elif op == "div":
            s = s / t(scale)
        if g == 0:
            acc = (np.zeros(out_shape, x.dtype) + s) if init_zero else s
        else:
            acc = acc + s
    return acc


def fold_values(tap_values, terms, init_zero=False, dtype=np.float32) -> np.ndarray:
    """The program's fold over already gathered tap values: tap_values[k] holds the values of
    the program's k-th tap (terms' taps in order) at a set of output points."""
    t = np.dtype(dtype).type
    k = 0
    acc = None
    for g, (op, scale, taps) in enumerate(terms):
        s = np.array(tap_values[k], dtype=dtype, copy=True)
        k += 1
        for _ in taps[1:]:
            s = s + tap_values[k]
            k += 1
        if op == "mul":
            s = t(scale) * s
        elif op == "div":
            s = s / t(scale)
        if g == 0:
            acc = (np.zeros(s.shape, dtype) + s) if init_zero else s
        else:
            acc = acc + s
    return acc


def eval_program_at(x: np.ndarray, points: np.ndarray, terms, init_zero=False, boundary="zero", shrink=()) -> np.ndarray:
    """Program value at output indices `points` (shape [k, ndim]) — for full-size grids,
    where only a sample of outputs can be re-computed on the host."""
    t = x.dtype.type
    nd = x.ndim
    pts = np.asarray(points, dtype=np.int64)

    def tap(o):
        idx = pts + np.asarray(o, dtype=np.int64)[None, :]
        ok = np.ones(len(pts), bool)
        for a in range(nd):
            ok &= (idx[:, a] >= 0) & (idx[:, a] < x.shape[a])
        vals = np.zeros(len(pts), x.dtype)
        sel = tuple(idx[ok, a] for a in range(nd))
        vals[ok] = x[sel]
        return vals

    acc = None
    for g, (op, scale, taps) in enumerate(terms):
        s = tap(taps[0]).copy()
        for o in taps[1:]:
            s = s + tap(o)
        if op == "mul":
            s = t(scale) * s
        elif op == "div":
            s = s / t(scale)
        if g == 0:
            acc = (np.zeros(len(pts), x.dtype) + s) if init_zero else s
        else:
            acc = acc + s
    return acc


def box_terms(ndim: int, radius: int, coeffs=None, descending=False):
    """Terms of the reference's box operator (flir_builder.rs:58-65, executor.rs:207-289)."""
    w = 2 * radius + 1
    n = w ** ndim
    terms = []
    for k in range(n):
        o, r = [], k
        for _ in range(ndim):
            o.append(r % w - radius)
            r //= w
        o = tuple(reversed(o))
        if descending:
            o = tuple(-v for v in o)
        terms.append(("mul", float(coeffs[k]) if coeffs is not None else 1.0 / n, (o,)))
    return terms


def sweeps(x: np.ndarray, fn, n: int) -> np.ndarray:
    for _ in range(n):
        x = fn(x)
    return x
