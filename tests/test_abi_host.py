"""The C ABI without a GPU: exports, host-side logic and argument checking.

Nothing here launches a kernel; calls that would reach the GPU are only made with
arguments the library must reject before touching CUDA.
"""
import ctypes
import re
import subprocess
from pathlib import Path

import pytest

from basalto import _abi, program as P

REPO = Path(__file__).resolve().parent.parent
HEADER = REPO / "include" / "basalto_b200.h"


def _declared():
    txt = HEADER.read_text()
    return sorted(set(re.findall(r"^BST_API\s+[\w\s\*]+?\b(bst_\w+)\s*\(", txt, re.M)))


def test_library_exports_every_declared_symbol():
    names = _declared()
    assert len(names) >= 25
    out = subprocess.run(["nm", "-D", "--defined-only", str(_abi.LIB_PATH)], capture_output=True, text=True).stdout
    exported = {ln.split()[-1] for ln in out.splitlines() if ln.strip()}
    missing = [n for n in names if n not in exported]
    assert not missing, missing
    # Nothing beyond the C ABI leaks out of the library.
    assert all(e.startswith("bst_") for e in exported), sorted(e for e in exported if not e.startswith("bst_"))
    lib = _abi.lib()
    for n in names:
        assert hasattr(lib, n)
    assert {s[0] for s in _abi.SIGNATURES} == set(names)


def test_rust_extension_surface():
    from basalto import _rust
    it = _rust.PyBasaltoInterceptor()
    assert hasattr(it, "compile_and_execute")
    assert _rust.abi_version() == 1
    assert _rust.PROGRAM_NBYTES == ctypes.sizeof(_abi.CProgram)


@pytest.mark.parametrize("op,r", [
    ("stencil", 1), ("stencil_r3", 3), ("stencil_r12", 12), ("stencil_r3_r4", 3), ("_r7", 7),
    ("stencil_r", 1), ("stencil_rx", 1), ("foo_order_8", 4), ("order_12", 6), ("a_r5order_8", 4),
])
def test_extract_radius_follows_interceptor_rules(op, r):
    """interceptor.rs:196-205: split('_r').nth(1).parse(), else order_8 -> 4, order_12 -> 6, else 1."""
    assert _abi.lib().bst_extract_radius(op.encode()) == r


def test_program_box_matches_python_builder():
    lib = _abi.lib()
    for ndim, r in [(1, 1), (2, 2), (3, 1), (3, 4)]:
        cp = _abi.CProgram()
        _abi.check(lib.bst_program_box(ndim, r, None, 0, ctypes.byref(cp)))
        py = P.box(ndim, r).to_c()
        assert bytes(cp) == bytes(py), (ndim, r)
    cp = _abi.CProgram()
    assert lib.bst_program_box(3, 1, (ctypes.c_double * 5)(), 5, ctypes.byref(cp)) == _abi.BST_ERR_INVALID
    assert lib.bst_program_box(3, 7, None, 0, ctypes.byref(cp)) == _abi.BST_ERR_UNSUPPORTED


def _b3(data: bytes, key=None):
    out = (ctypes.c_uint8 * 32)()
    buf = (ctypes.c_uint8 * max(len(data), 1)).from_buffer_copy(data or b"\0")
    kb = (ctypes.c_uint8 * 32).from_buffer_copy(key) if key else None
    _abi.check(_abi.lib().bst_blake3(buf, len(data), kb, out))
    return bytes(out).hex()


def test_blake3_published_vectors():
    """Known answers of the BLAKE3 specification (input bytes i % 251; key
    'whats the Elvish word for friend'), covering one block, one chunk and the tree."""
    inp = lambda n: bytes(i % 251 for i in range(n))  # noqa: E731
    key = b"whats the Elvish word for friend"
    assert _b3(inp(0)) == "af1349b9f5f9a1a6a0404dea36dcc9499bcb25c9adc112b7cc9a93cae41f3262"
    assert _b3(inp(1)) == "2d3adedff11b61f14c886e35afa036736dcd87a74d27b5c1510225d0f592e213"
    assert _b3(inp(1024)) == "42214739f095a406f3fc83deb889744ac00df831c10daa55189b5d121c855af7"
    assert _b3(inp(1025)) == "d00278ae47eb27b34faecf67b4fe263f82d5412916c1ffd97c8cb7fb814b8444"
    assert _b3(inp(8193)) == "bab6c09cb8ce8cf459261398d2e7aef35700bf488116ceb94a36d0f5f1b7bc3b"
    assert _b3(inp(0), key).startswith("92b2b75604ed3c761f9d6f62392c8a9227ad0ea3f09573e783f1498a4ed60d26"[:16])


def _serialize(op, dtype, shape, strides, radius, caps):
    """Python restatement of hasher.rs:53-121 (stencil path: no matmul fields)."""
    def fixed(s, w):
        b = s.encode()[:w]
        return b + b"\0" * (w - len(b))
    b = fixed(op, 32) + fixed(dtype, 16)
    b += len(shape).to_bytes(8, "little") + b"".join(int(s).to_bytes(8, "little") for s in shape)
    b += len(strides).to_bytes(8, "little") + b"".join(int(s).to_bytes(8, "little", signed=True) for s in strides)
    b += int(radius).to_bytes(8, "little") + b"\0"
    b += fixed(caps["vendor"], 16) + fixed(caps["arch"], 16) + fixed(caps["driver"], 32)
    for k, w in [("compute_capability_major", 4), ("compute_capability_minor", 4), ("max_threads_per_block", 4),
                 ("max_shared_memory_per_block", 8), ("max_registers_per_block", 4), ("warp_size", 4),
                 ("multi_processor_count", 4)]:
        b += int(caps[k]).to_bytes(w, "little", signed=(w == 4))
    return b


def test_cache_key_layout_and_sensitivity():
    from basalto import api
    caps = {"compute_capability_major": 10, "compute_capability_minor": 0, "max_threads_per_block": 1024,
            "max_shared_memory_per_block": 49152, "max_registers_per_block": 65536, "warp_size": 32,
            "multi_processor_count": 148, "name": "B200", "vendor": "nvidia", "arch": "sm_100",
            "driver": "580.159", "driver_version": 12090}
    key = bytes(range(32))
    k = api.cache_key("stencil", "float32", [8, 9, 10], [90, 10, 1], 1, caps, key=key)
    ser = _serialize("stencil", "float32", [8, 9, 10], [90, 10, 1], 1, caps)
    assert k == _b3(ser, key)
    assert len(k) == 64
    assert api.cache_key("stencil", "float32", [8, 9, 10], [90, 10, 1], 2, caps, key=key) != k
    assert api.cache_key("stencil", "float64", [8, 9, 10], [90, 10, 1], 1, caps, key=key) != k
    assert api.cache_key("stencil", "float32", [8, 9, 10], [90, 10, 1], 1, caps, extra=b"P", key=key) != k
    # No capabilities: 56 zero bytes in their place (hasher.rs:116-118).
    none = api.cache_key("stencil", "float32", [4], [1], 1, None, key=key)
    ser = _serialize("stencil", "float32", [4], [1], 1, dict(caps, vendor="unknown", arch="generic", driver="unknown"))
    ser = ser[:-(4 * 6 + 8)] + b"\0" * 56
    assert none == _b3(ser, key)


def _apply(prog_c, ndim, shape, x=1, y=2):
    lib = _abi.lib()
    return lib.bst_stencil_apply(ctypes.byref(prog_c), _abi.BST_F32, ndim, _abi.i64_array(shape), None,
                                 ctypes.c_void_p(x), None, ctypes.c_void_p(y), None)


def test_apply_rejects_bad_programs_before_any_device_work():
    cp = P.heat7_3d().to_c()
    assert _apply(cp, 3, [4, 4, 4], x=0, y=0) == _abi.BST_ERR_INVALID        # null pointers
    assert _apply(cp, 2, [4, 4]) == _abi.BST_ERR_INVALID                      # ndim mismatch
    assert _apply(cp, 4, [4, 4, 4, 4]) == _abi.BST_ERR_INVALID                # rank 4
    bad = P.heat7_3d().to_c()
    bad.term_first[1] = 2                                                     # gap in the partition
    assert _apply(bad, 3, [4, 4, 4]) == _abi.BST_ERR_INVALID
    bad = P.heat7_3d().to_c()
    bad.term_op[0] = 7
    assert _apply(bad, 3, [4, 4, 4]) == _abi.BST_ERR_INVALID
    assert b"operator" in _abi.lib().bst_last_error()
    v = P.mean3_1d().to_c([10])
    v.out_shape[0] = 9                                                        # reads past the end
    assert _apply(v, 1, [10]) == _abi.BST_ERR_INVALID
    assert _apply(P.heat7_3d().to_c(), 3, [0, 4, 4], x=0, y=0) == _abi.BST_OK  # empty grid: no-op
    lib = _abi.lib()
    assert lib.bst_stencil_apply(ctypes.byref(cp), 5, 3, _abi.i64_array([4, 4, 4]), None, ctypes.c_void_p(1),
                                 None, ctypes.c_void_p(2), None) == _abi.BST_ERR_UNSUPPORTED
    bad = P.heat7_3d().to_c()
    bad.flags = 6                                                             # only BST_PROGRAM_CONTRACT exists
    assert _apply(bad, 3, [4, 4, 4]) == _abi.BST_ERR_INVALID
    assert b"flags" in lib.bst_last_error()
    fused = P.heat7_3d().contracted().to_c()
    assert fused.flags == _abi.BST_PROGRAM_CONTRACT
    # the allocation-free entry point does not take fused multiply-add programs
    assert lib.bst_stencil_apply_noalloc(ctypes.byref(fused), 0, 3, _abi.i64_array([4, 4, 4]), None,
                                         ctypes.c_void_p(16), None, ctypes.c_void_p(32),
                                         None) == _abi.BST_ERR_UNSUPPORTED


def test_interceptor_rejects_like_the_reference():
    lib = _abi.lib()
    h = ctypes.c_void_p()
    _abi.check(lib.bst_interceptor_create(ctypes.byref(h)))
    try:
        sh, st = _abi.i64_array([2, 2, 2, 2]), _abi.i64_array([8, 4, 2, 1])
        rc = lib.bst_interceptor_compile_and_execute(h, b"stencil", b"float32", 4, sh, st, None, 1, 2, 0, None, 0,
                                                     None, None)
        assert rc == _abi.BST_ERR_INVALID
        rc = lib.bst_interceptor_compile_and_execute(h, b"matmul", b"float32", 3, sh, st, None, 1, 2, 3, None, 0,
                                                     None, None)
        assert rc == _abi.BST_ERR_UNSUPPORTED
        rc = lib.bst_interceptor_compile_and_execute(h, b"stencil", b"float32", 2, sh, st, None, 0, 0, 0, None, 0,
                                                     None, None)
        assert rc == _abi.BST_ERR_INVALID
        rc = lib.bst_interceptor_compile_and_execute(h, b"stencil", b"int8", 2, sh, st, None, 1, 2, 0, None, 0,
                                                     None, None)
        assert rc == _abi.BST_ERR_UNSUPPORTED
        assert lib.bst_interceptor_cache_size(h) == 0
    finally:
        lib.bst_interceptor_destroy(h)


def test_comm_arguments_checked_on_host():
    lib = _abi.lib()
    h = ctypes.c_void_p()
    uid = (ctypes.c_uint8 * 128)()
    assert lib.bst_comm_create(uid, 2, 5, 0, 1.0, ctypes.byref(h)) == _abi.BST_ERR_INVALID
    assert lib.bst_halo_exchange(None, None, 0, 1, 1, 1, None) == _abi.BST_ERR_INVALID
    assert lib.bst_comm_rank(None) == -1 and lib.bst_comm_size(None) == -1
