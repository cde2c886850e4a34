"""ctypes view of the C ABI in include/basalto_b200.h (libbasalto_b200.so).

The library is loaded from this package directory.  The `basalto._rust` extension links
the same file, so both see one library instance (one launch counter, one plan cache per
interceptor).  Loading fails loudly when the library has not been built.
"""
from __future__ import annotations

import ctypes
from ctypes import c_char_p, c_double, c_int32, c_int64, c_uint8, c_uint64, c_void_p, POINTER
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libbasalto_b200.so"

MAX_TAPS = 2304
MAX_TERMS = 2304

BST_OK, BST_ERR_INVALID, BST_ERR_UNSUPPORTED, BST_ERR_CUDA, BST_ERR_NCCL, BST_ERR_TIMEOUT, BST_ERR_NO_DEVICE = range(7)
BST_F32, BST_F64 = 0, 1
BST_PROGRAM_CONTRACT = 1  # program flag: fold later multiplied terms with fma
TERM_SUM, TERM_MUL, TERM_DIV = 0, 1, 2
BOUNDARY_ZERO, BOUNDARY_VALID = 0, 1


class CProgram(ctypes.Structure):
    _fields_ = [
        ("ndim", c_int32),
        ("ntaps", c_int32),
        ("nterms", c_int32),
        ("init_zero", c_int32),
        ("boundary", c_int32),
        ("flags", c_int32),
        ("out_shape", c_int64 * 3),
        ("tap", (c_int32 * 3) * MAX_TAPS),
        ("term_first", c_int32 * MAX_TERMS),
        ("term_count", c_int32 * MAX_TERMS),
        ("term_op", c_int32 * MAX_TERMS),
        ("term_scale", c_double * MAX_TERMS),
    ]


class CDeviceCaps(ctypes.Structure):
    _fields_ = [
        ("compute_capability_major", c_int32),
        ("compute_capability_minor", c_int32),
        ("max_threads_per_block", c_int32),
        ("max_shared_memory_per_block", c_uint64),
        ("max_registers_per_block", c_int32),
        ("warp_size", c_int32),
        ("multi_processor_count", c_int32),
        ("name", ctypes.c_char * 96),
        ("vendor", ctypes.c_char * 16),
        ("arch", ctypes.c_char * 16),
        ("driver", ctypes.c_char * 32),
        ("driver_version", c_int32),
    ]


# (name, restype, argtypes) for every entry point of include/basalto_b200.h
SIGNATURES = [
    ("bst_abi_version", c_int32, []),
    ("bst_last_error", c_char_p, []),
    ("bst_launch_count", c_uint64, []),
    ("bst_device_error_check", c_int32, [c_void_p]),
    ("bst_program_box", c_int32, [c_int32, c_int32, POINTER(c_double), c_int64, POINTER(CProgram)]),
    ("bst_extract_radius", c_int32, [c_char_p]),
    ("bst_stencil_apply", c_int32,
     [POINTER(CProgram), c_int32, c_int32, POINTER(c_int64), POINTER(c_int64), c_void_p, POINTER(c_int64),
      c_void_p, c_void_p]),
    ("bst_stencil_apply_noalloc", c_int32,
     [POINTER(CProgram), c_int32, c_int32, POINTER(c_int64), POINTER(c_int64), c_void_p, POINTER(c_int64),
      c_void_p, c_void_p]),
    ("bst_stencil_sweeps", c_int32,
     [POINTER(CProgram), c_int32, c_int32, POINTER(c_int64), c_void_p, c_void_p, c_int32, c_void_p]),
    ("bst_stencil_sweeps_fused", c_int32,
     [POINTER(CProgram), c_int32, c_int32, POINTER(c_int64), c_void_p, c_void_p, c_int32, c_int32, c_void_p]),
    ("bst_device_caps_query", c_int32, [c_int32, POINTER(CDeviceCaps)]),
    ("bst_cache_key", c_int32,
     [c_char_p, c_char_p, c_int32, POINTER(c_int64), POINTER(c_int64), c_int64, POINTER(CDeviceCaps),
      POINTER(c_uint8), c_int64, POINTER(c_uint8), ctypes.c_char_p]),
    ("bst_blake3", c_int32, [POINTER(c_uint8), c_int64, POINTER(c_uint8), POINTER(c_uint8)]),
    ("bst_interceptor_create", c_int32, [POINTER(c_void_p)]),
    ("bst_interceptor_destroy", None, [c_void_p]),
    ("bst_interceptor_compile_and_execute", c_int32,
     [c_void_p, c_char_p, c_char_p, c_int32, POINTER(c_int64), POINTER(c_int64), c_char_p, c_uint64, c_uint64,
      c_uint64, POINTER(c_double), c_int64, POINTER(CProgram), c_void_p]),
    ("bst_interceptor_cache_size", c_int64, [c_void_p]),
    ("bst_interceptor_cache_hits", c_int64, [c_void_p]),
    ("bst_interceptor_last_key", c_int32, [c_void_p, ctypes.c_char_p]),
    ("bst_nccl_get_unique_id", c_int32, [POINTER(c_uint8)]),
    ("bst_comm_create", c_int32, [POINTER(c_uint8), c_int32, c_int32, c_int32, c_double, POINTER(c_void_p)]),
    ("bst_comm_destroy", c_int32, [c_void_p]),
    ("bst_comm_abort", c_int32, [c_void_p]),
    ("bst_comm_rank", c_int32, [c_void_p]),
    ("bst_comm_size", c_int32, [c_void_p]),
    ("bst_halo_exchange", c_int32, [c_void_p, c_void_p, c_int32, c_int64, c_int64, c_int32, c_void_p]),
    ("bst_slab_sweeps", c_int32,
     [c_void_p, POINTER(CProgram), c_int32, c_int32, POINTER(c_int64), c_void_p, c_void_p, c_int32, c_void_p]),
    ("bst_slab_ghost_depth", c_int32, [POINTER(CProgram), c_int32, c_int32, POINTER(c_int64), POINTER(c_int32)]),
    ("bst_slab_sweeps_deep", c_int32,
     [c_void_p, POINTER(CProgram), c_int32, c_int32, POINTER(c_int64), c_int32, c_void_p, c_void_p, c_int32,
      c_void_p]),
    ("bst_comm_register_slab", c_int32, [c_void_p, c_void_p, c_int32, c_int64, c_int64, c_int32]),
    ("bst_slab_sweeps_p2p", c_int32,
     [c_void_p, POINTER(CProgram), c_int32, c_int32, POINTER(c_int64), c_int32, c_void_p, c_void_p, c_int32,
      c_void_p]),
    ("bst_slab_sweeps_copy", c_int32,
     [c_void_p, POINTER(CProgram), c_int32, c_int32, POINTER(c_int64), c_int32, c_void_p, c_void_p, c_int32,
      c_void_p]),
    ("bst_comm_profile_begin", c_int32, [c_void_p, c_int32]),
    ("bst_march_item_plan", c_int32, [c_int64, c_int64, c_int32, c_int32, c_int64, POINTER(c_int64)]),
    ("bst_comm_profile_end", c_int32, [c_void_p, POINTER(c_double)]),
]

_lib = None


class BasaltoError(RuntimeError):
    """A C-ABI call returned a non-zero bst_status."""

    def __init__(self, code: int, msg: str):
        super().__init__(msg)
        self.code = code


def lib():
    """The loaded C-ABI library (raises OSError if it was never built)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise OSError(f"{LIB_PATH} is missing: build it with bs-compiler_b200/csrc/build.py")
        h = ctypes.CDLL(str(LIB_PATH))
        for name, res, args in SIGNATURES:
            fn = getattr(h, name)
            fn.restype = res
            fn.argtypes = args
        _lib = h
    return _lib


def check(rc: int) -> None:
    if rc != BST_OK:
        raise BasaltoError(rc, lib().bst_last_error().decode(errors="replace"))


def i64_array(values) -> ctypes.Array:
    vals = list(values)
    return (c_int64 * max(len(vals), 1))(*vals)
