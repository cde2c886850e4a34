"""bst_stencil_apply_noalloc: the sweep for callers that cannot allocate GPU memory.

Some callers must not allocate device memory while they run (a real-time loop with a fixed
memory budget, a framework that owns every device byte through its own pool, code that
cannot afford cudaMalloc's implicit synchronisation).  For them the library keeps the
runtime-table kernel's table in a fixed 32 KiB device array instead of a per-call buffer.
These tests call that entry point through the C ABI and require its output to equal the
general entry point's (bst_stencil_apply) and the CPU oracle's bit for bit — the tolerance of
every other kernel test here — on consecutive calls with different programs, so each call
must fully replace what the previous one left in the shared array.  They also check that a
call leaves the device's memory untouched: no pool allocation (the default pool's high-water
mark) and no lasting allocation (free device memory).  Collected last on purpose.
"""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _lib():
    from basalto import _abi
    return _abi


def _call(entry, prog, x, out):
    A = _lib()
    cp = prog.to_c(x.shape)
    fn = getattr(A.lib(), entry)
    rc = fn(ctypes.byref(cp), A.BST_F32 if x.dtype == torch.float32 else A.BST_F64, x.dim(),
            A.i64_array(x.shape), A.i64_array(x.stride()), ctypes.c_void_p(x.data_ptr()),
            A.i64_array(out.stride()), ctypes.c_void_p(out.data_ptr()),
            ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    return rc


def _both(prog, x):
    """(general entry point, allocation-free entry point), after checking the latter against
    the CPU oracle."""
    from oracle import stencil_oracle as O
    A = _lib()
    shape = prog.out_shape(x.shape)
    ref = torch.full(shape, float("nan"), dtype=x.dtype, device=x.device)
    got = torch.full(shape, float("nan"), dtype=x.dtype, device=x.device)
    A.check(_call("bst_stencil_apply", prog, x, ref))
    A.check(_call("bst_stencil_apply_noalloc", prog, x, got))
    torch.cuda.synchronize()
    want = O.eval_program(x.cpu().numpy(), [(t.op, t.scale, t.taps) for t in prog.terms], prog.init_zero,
                          prog.boundary, prog.shrink)
    assert np.array_equal(got.cpu().numpy(), want)
    return ref.cpu().numpy(), got.cpu().numpy()


class _Driver:
    """The CUDA driver API through ctypes: the device's default memory pool and free memory."""

    USED_MEM_HIGH = 8  # CU_MEMPOOL_ATTR_USED_MEM_HIGH

    def __init__(self):
        self.cu = ctypes.CDLL("libcuda.so.1")
        dev = ctypes.c_int(0)
        assert self.cu.cuDeviceGet(ctypes.byref(dev), torch.cuda.current_device()) == 0
        self.pool = ctypes.c_void_p()
        assert self.cu.cuDeviceGetDefaultMemPool(ctypes.byref(self.pool), dev) == 0

    def pool_high(self):
        v = ctypes.c_uint64(0)
        assert self.cu.cuMemPoolGetAttribute(self.pool, self.USED_MEM_HIGH, ctypes.byref(v)) == 0
        return v.value

    def reset_pool_high(self):
        v = ctypes.c_uint64(0)
        assert self.cu.cuMemPoolSetAttribute(self.pool, self.USED_MEM_HIGH, ctypes.byref(v)) == 0

    def free_bytes(self):
        free, total = ctypes.c_size_t(0), ctypes.c_size_t(0)
        assert self.cu.cuMemGetInfo_v2(ctypes.byref(free), ctypes.byref(total)) == 0
        return free.value


def test_noalloc_matches_general_entry_point_on_consecutive_calls():
    from basalto import program as P
    from basalto.program import StencilProgram, Term

    g = torch.Generator().manual_seed(21)
    # First call: a 3-D program with two weighted terms (heat step), fp32.
    x1 = torch.rand(17, 24, 40, generator=g).cuda()
    r1, a1 = _both(P.heat7_3d(), x1)
    assert np.array_equal(r1, a1)
    # Second call: a different program (2-D radius-2 box, fp64, descending taps) and a
    # different grid; it must not see anything of the first call's table.
    x2 = torch.randn(33, 50, generator=g, dtype=torch.float64).cuda()
    w = (torch.rand(25, generator=g, dtype=torch.float64) - 0.5).tolist()
    r2, a2 = _both(P.box(2, 2, w, descending=True), x2)
    assert np.array_equal(r2, a2)
    # Third: a valid-region 1-D program with a division term (shrinking output).
    x3 = torch.randn(1001, generator=g).cuda()
    prog3 = StencilProgram(1, (Term("div", 3.0, ((0,), (1,), (2,))),), boundary="valid", shrink=(2,))
    r3, a3 = _both(prog3, x3)
    assert np.array_equal(r3, a3)


def test_noalloc_allocates_nothing():
    """After its first call on the device, a call neither raises the default pool's high-water
    mark (the general entry point allocates its runtime-table buffers there) nor holds device
    memory afterwards."""
    from basalto.program import StencilProgram, Term
    A = _lib()
    g = torch.Generator().manual_seed(4)
    x = torch.randn(23, 31, 47, generator=g).cuda()
    y = torch.empty_like(x)
    # a program outside the compiled catalog: the runtime-table kernel
    prog = StencilProgram(3, (Term("mul", 0.3, ((0, 0, 0), (1, 1, 0))), Term("div", 7.0, ((-1, 0, 2),)),
                              Term("sum", 0.0, ((0, -2, -1), (2, 0, 0)))))
    A.check(_call("bst_stencil_apply_noalloc", prog, x, y))  # first call: looks up the array's address
    torch.cuda.synchronize()
    drv = _Driver()
    drv.reset_pool_high()
    base_high = drv.pool_high()
    free0 = drv.free_bytes()
    torch_alloc0 = torch.cuda.memory_allocated()
    for _ in range(3):
        A.check(_call("bst_stencil_apply_noalloc", prog, x, y))
    torch.cuda.synchronize()
    assert drv.pool_high() == base_high
    assert drv.free_bytes() == free0
    assert torch.cuda.memory_allocated() == torch_alloc0


def test_noalloc_rejects_tables_beyond_its_array():
    A = _lib()
    from basalto import program as P

    prog = P.box(3, 6)  # 2197 taps: the packed table is far beyond 32 KiB
    x = torch.zeros(16, 16, 16, device="cuda")
    y = torch.empty_like(x)
    rc = _call("bst_stencil_apply_noalloc", prog, x, y)
    assert rc == A.BST_ERR_UNSUPPORTED
    assert "32768" in A.lib().bst_last_error().decode()
