"""Tensor-level entry points over the C ABI (include/basalto_b200.h)."""
from __future__ import annotations

import ctypes

import torch

from . import _abi
from .program import StencilProgram

_DT = {torch.float32: _abi.BST_F32, torch.float64: _abi.BST_F64}


def _stream_ptr(dev, stream=None):
    s = stream if stream is not None else torch.cuda.current_stream(dev)
    return ctypes.c_void_p(s.cuda_stream)


def _dtype(t: torch.Tensor) -> int:
    try:
        return _DT[t.dtype]
    except KeyError:
        raise TypeError(f"basalto stencils run in float32 or float64, got {t.dtype}") from None


def apply(prog: StencilProgram, x: torch.Tensor, out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
    """One sweep `out = prog(x)` on x's CUDA device and the current (or given) stream."""
    if not x.is_cuda:
        raise RuntimeError("basalto.apply needs a CUDA tensor")
    oshape = prog.out_shape(x.shape)
    if out is None:
        out = torch.empty(oshape, dtype=x.dtype, device=x.device)
    elif tuple(out.shape) != oshape or out.dtype != x.dtype or out.device != x.device:
        raise ValueError("out has the wrong shape, dtype or device")
    if out.numel() == 0:
        return out
    cp = prog.to_c(x.shape)
    with torch.cuda.device(x.device):
        _abi.check(_abi.lib().bst_stencil_apply(
            ctypes.byref(cp), _dtype(x), x.dim(), _abi.i64_array(x.shape), _abi.i64_array(x.stride()),
            ctypes.c_void_p(x.data_ptr()), _abi.i64_array(out.stride()), ctypes.c_void_p(out.data_ptr()),
            _stream_ptr(x.device, stream)))
    return out


def sweeps(prog: StencilProgram, a: torch.Tensor, b: torch.Tensor, nsteps: int, stream=None,
           max_fused: int = 0) -> torch.Tensor:
    """`nsteps` sweeps ping-ponging a -> b -> a ...; returns the buffer holding the result.
    max_fused > 0 fuses up to that many sweeps per launch wherever a temporally blocked kernel
    exists (0: the library's choice, which fuses only where that is faster)."""
    if not (a.is_cuda and b.is_cuda):
        raise RuntimeError("basalto.sweeps needs CUDA tensors")
    if a.shape != b.shape or a.dtype != b.dtype or not (a.is_contiguous() and b.is_contiguous()):
        raise ValueError("ping-pong buffers must be contiguous tensors of one shape and dtype")
    cp = prog.to_c(a.shape)
    with torch.cuda.device(a.device):
        _abi.check(_abi.lib().bst_stencil_sweeps_fused(
            ctypes.byref(cp), _dtype(a), a.dim(), _abi.i64_array(a.shape), ctypes.c_void_p(a.data_ptr()),
            ctypes.c_void_p(b.data_ptr()), int(nsteps), int(max_fused), _stream_ptr(a.device, stream)))
    return b if nsteps % 2 else a


def check_device_errors(device=None) -> None:
    """Raise if a kernel on `device` gave up a bounded wait since the last check."""
    dev = torch.device("cuda", torch.cuda.current_device() if device is None else device)
    with torch.cuda.device(dev):
        _abi.check(_abi.lib().bst_device_error_check(_stream_ptr(dev)))


def launch_count() -> int:
    """Kernels launched by the native library in this process."""
    return int(_abi.lib().bst_launch_count())


def device_caps(device: int = 0) -> dict:
    c = _abi.CDeviceCaps()
    _abi.check(_abi.lib().bst_device_caps_query(device, ctypes.byref(c)))
    return {k: (getattr(c, k).decode() if isinstance(getattr(c, k), bytes) else getattr(c, k))
            for k, _ in _abi.CDeviceCaps._fields_}


def cache_key(op: str, dtype: str, shape, strides, radius: int, caps: dict | None = None,
              extra: bytes = b"", key: bytes | None = None) -> str:
    """The interceptor's cache key (hasher.rs serialization, keyed BLAKE3) as 64 hex chars."""
    cp = None
    if caps is not None:
        cp = _abi.CDeviceCaps()
        for k, _ in _abi.CDeviceCaps._fields_:
            v = caps[k]
            setattr(cp, k, v.encode() if isinstance(v, str) else v)
    ex = (ctypes.c_uint8 * max(len(extra), 1)).from_buffer_copy(extra or b"\0")
    kb = (ctypes.c_uint8 * 32).from_buffer_copy(key) if key is not None else None
    out = ctypes.create_string_buffer(65)
    _abi.check(_abi.lib().bst_cache_key(op.encode(), dtype.encode(), len(shape), _abi.i64_array(shape),
                                        _abi.i64_array(strides), int(radius),
                                        ctypes.byref(cp) if cp is not None else None, ex, len(extra), kb, out))
    return out.value.decode()
