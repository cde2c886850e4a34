"""CPU oracle for the stencil hot path — TEST INFRASTRUCTURE ONLY.

Imported by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg as the checker;
never by the product path (the `basalto` package does not import this package).
"""
from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
C_LIB = HERE / "_build" / "liboracle.so"

_c = None


def build_c() -> Path:
    """Compile naive_stencil.c with the committed Makefile (gcc)."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return C_LIB


def c_oracle():
    global _c
    if _c is None:
        if not C_LIB.exists() or C_LIB.stat().st_mtime < (HERE / "naive_stencil.c").stat().st_mtime:
            build_c()
        _c = ctypes.CDLL(str(C_LIB))
    return _c


def _i64(v):
    return (ctypes.c_int64 * max(len(v), 1))(*[int(s) for s in v])


def naive_box_f64(x: np.ndarray, radius: int, coeffs) -> np.ndarray:
    """executor.rs:207-289 restated in C (float64, C-contiguous layout)."""
    x = np.ascontiguousarray(x, dtype=np.float64)
    out = np.empty_like(x)
    c = np.ascontiguousarray(coeffs, dtype=np.float64)
    c_oracle().oracle_naive_box_f64(x.ctypes.data_as(ctypes.c_void_p), out.ctypes.data_as(ctypes.c_void_p),
                                    x.ndim, _i64(x.shape), radius, c.ctypes.data_as(ctypes.c_void_p))
    return out


def program_c(x: np.ndarray, terms, init_zero=False, boundary="zero", shrink=(), contract=False) -> np.ndarray:
    """Point-by-point C evaluation of a program (terms = [(op, scale, taps), ...]); with
    `contract`, later multiplied terms fold as acc = fma(scale, sum, acc)."""
    x = np.ascontiguousarray(x)
    nd = x.ndim
    out_shape = x.shape if boundary == "zero" else tuple(x.shape[a] - shrink[a] for a in range(nd))
    out = np.empty(out_shape, x.dtype)
    ops = {"sum": 0, "mul": 1, "div": 2}
    op = np.array([ops[t[0]] for t in terms], np.int32)
    sc = np.array([float(t[1]) for t in terms], np.float64)
    cnt = np.array([len(t[2]) for t in terms], np.int32)
    taps = np.array([list(o) + [0] * (3 - nd) for t in terms for o in t[2]], np.int32).reshape(-1)
    fn = c_oracle().oracle_program_f32 if x.dtype == np.float32 else c_oracle().oracle_program_f64
    p = lambda a: a.ctypes.data_as(ctypes.c_void_p)  # noqa: E731
    fn(p(x), p(out), nd, _i64(x.shape), 0 if boundary == "zero" else 1, _i64(out_shape), int(bool(init_zero)),
       len(terms), p(op), p(sc), p(cnt), p(taps), int(bool(contract)))
    return out
