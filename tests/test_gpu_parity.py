"""GPU parity: the sm_100a kernels against the oracle and the golden fixtures, bit for bit.

Every comparison is np.array_equal (exact): the kernels perform the same separately rounded
operations in the same order as eager torch.
"""
import ctypes

import numpy as np
import pytest
import torch

from conftest import Golden, GOLDEN, program_from_meta, oracle_terms
from oracle import stencil_oracle as O
import oracle

pytestmark = pytest.mark.gpu

G = Golden(GOLDEN)
NAMES = sorted(G.cases)


def _basalto():
    import basalto
    return basalto


def _run_steps(fn, x, steps):
    for _ in range(steps):
        x = fn(x)
    return x


@pytest.mark.parametrize("name", NAMES)
def test_golden_via_c_abi(name):
    b = _basalto()
    case = G.cases[name]
    prog = program_from_meta(case["program"])
    x = torch.from_numpy(G.input(name)).cuda()
    n0 = b.launch_count()
    y = _run_steps(lambda u: b.apply(prog, u), x, case["steps"])
    torch.cuda.synchronize()
    assert np.array_equal(y.cpu().numpy(), G.output(name))
    if y.numel():
        assert b.launch_count() > n0  # the native kernels ran


@pytest.mark.parametrize("name", NAMES)
def test_golden_via_interceptor(name):
    b = _basalto()
    case = G.cases[name]
    prog = program_from_meta(case["program"])
    it = b._rust.PyBasaltoInterceptor()
    x = torch.from_numpy(G.input(name)).cuda()
    for _ in range(case["steps"]):
        y = torch.empty(prog.out_shape(x.shape), dtype=x.dtype, device="cuda")
        if y.numel():
            it.compile_and_execute("stencil", str(x.dtype).split(".")[-1], list(x.shape), list(x.stride()), None,
                                   x.data_ptr(), y.data_ptr(), 0, program=prog.pack(x.shape))
        x = y
    assert np.array_equal(x.cpu().numpy(), G.output(name))


WORKLOAD_CASES = [n for n in NAMES if not n.startswith("ref_")]


@pytest.mark.parametrize("name", WORKLOAD_CASES)
def test_golden_via_torch_compile(name):
    b = _basalto()
    from basalto import workloads as W
    case = G.cases[name]
    kind = name.split("_")[0] + "_" + name.split("_")[1]
    fn = {"mean3_1d": W.mean3_1d, "jacobi5_2d": W.jacobi5_2d, "heat7_3d": W.heat7_3d,
          "box27_3d": W.make_box27_3d(case.get("weights") or W.box27_weights()),
          "star25_3d": W.make_star_3d()}[kind]
    torch._dynamo.reset()
    cf = torch.compile(fn, backend="basalto")
    x = torch.from_numpy(G.input(name)).cuda()
    n0 = b.launch_count()
    y = _run_steps(cf, x, case["steps"])
    torch.cuda.synchronize()
    assert y.is_cuda
    assert np.array_equal(y.cpu().numpy(), G.output(name))
    if y.numel():
        assert b.launch_count() >= n0 + case["steps"]


# ---- shapes beyond the fixtures: TMA-eligible and ragged sizes, both dtypes -------------

SHAPES_2D = [(1, 4), (2, 8), (17, 64), (33, 128), (257, 512), (100, 1000), (129, 260), (7, 13)]
SHAPES_3D = [(3, 4, 8), (17, 33, 64), (9, 40, 128), (5, 7, 256), (33, 17, 100), (4, 5, 6), (70, 3, 36)]


def _workload_programs():
    from basalto import program as P
    from basalto import workloads as W
    return {
        "jacobi5_2d": (P.jacobi5_2d(), 2),
        "box2d_r1": (P.box(2, 1), 2),
        "box2d_r3": (P.box(2, 3), 2),
        "heat7_3d": (P.heat7_3d(), 3),
        "box27_3d": (P.box(3, 1, W.box27_weights()), 3),
        "star25_3d": (P.star_3d(P.LAPLACIAN8_COEFFS), 3),
        "box3d_r2": (P.box(3, 2), 3),
        "box3d_r1_desc": (P.box(3, 1, descending=True), 3),
    }


@pytest.mark.parametrize("dtype", [torch.float32, torch.float64])
@pytest.mark.parametrize("key", list(_workload_programs()))
def test_kernels_vs_oracle_many_shapes(key, dtype):
    b = _basalto()
    prog, nd = _workload_programs()[key]
    shapes = SHAPES_2D if nd == 2 else SHAPES_3D
    g = torch.Generator().manual_seed(11)
    for shape in shapes:
        x = torch.randn(shape, generator=g, dtype=dtype)
        ref = O.eval_program(x.numpy(), oracle_terms(prog), prog.init_zero)
        got = b.apply(prog, x.cuda()).cpu().numpy()
        assert np.array_equal(got, ref), f"{key} {shape} {dtype}"


@pytest.mark.parametrize("dtype", [torch.float32, torch.float64])
def test_strided_inputs_take_the_general_path(dtype):
    b = _basalto()
    from basalto import program as P
    g = torch.Generator().manual_seed(12)
    base = torch.randn(40, 50, 60, generator=g, dtype=dtype)
    for view in (base[:, 1:-1, 3:], base.transpose(1, 2), base[::2]):
        prog = P.heat7_3d()
        ref = O.eval_program(np.ascontiguousarray(view.numpy()), oracle_terms(prog))
        got = b.apply(prog, view.cuda() if view.is_contiguous() else base.cuda().as_strided(view.shape, view.stride(), view.storage_offset()))
        assert np.array_equal(got.cpu().numpy(), ref)


@pytest.mark.parametrize("ndim,radius", [(1, 1), (1, 2), (1, 4), (1, 6), (2, 1), (2, 2), (2, 4), (2, 5), (3, 1), (3, 2), (3, 3)])
def test_reference_operator_isotropic_box(ndim, radius):
    """compile_and_execute("stencil_r<k>") without a program: the reference's operator —
    isotropic (2r+1)^d box, zero padded, accumulated from 0 in ascending offset order."""
    b = _basalto()
    shape = {1: (1000,), 2: (37, 64), 3: (11, 13, 24)}[ndim]
    g = torch.Generator().manual_seed(13)
    for dtype in (torch.float32, torch.float64):
        x = torch.randn(shape, generator=g, dtype=dtype)
        xd = x.cuda()
        y = torch.zeros_like(xd)
        it = b._rust.PyBasaltoInterceptor()
        op = f"stencil_r{radius}"
        it.compile_and_execute(op, str(dtype).split(".")[-1], list(x.shape), list(x.stride()), None,
                               xd.data_ptr(), y.data_ptr(), 0)
        ref = O.eval_program(x.numpy(), O.box_terms(ndim, radius), init_zero=True)
        assert np.array_equal(y.cpu().numpy(), ref), (ndim, radius, dtype)
        if dtype == torch.float64:
            n = (2 * radius + 1) ** ndim
            assert np.array_equal(y.cpu().numpy(), oracle.naive_box_f64(x.numpy(), radius, [1.0 / n] * n))


def test_reference_operator_order_names_and_cache():
    b = _basalto()
    it = b._rust.PyBasaltoInterceptor()
    x = torch.randn(9, 10, 12, dtype=torch.float64, device="cuda")
    y = torch.empty_like(x)
    for op, r in (("stencil", 1), ("stencil_order_8", 4)):
        if r > 3:  # 3-D radius 4 is 729 taps: covered in 2-D; use a 2-D grid here
            x2 = torch.randn(20, 24, dtype=torch.float64, device="cuda")
            y2 = torch.empty_like(x2)
            it.compile_and_execute(op, "f64", list(x2.shape), list(x2.stride()), "job", x2.data_ptr(), y2.data_ptr(), 0)
            ref = O.eval_program(x2.cpu().numpy(), O.box_terms(2, 4), init_zero=True)
            assert np.array_equal(y2.cpu().numpy(), ref)
        else:
            it.compile_and_execute(op, "float64", list(x.shape), list(x.stride()), None, x.data_ptr(), y.data_ptr(), 0)
            ref = O.eval_program(x.cpu().numpy(), O.box_terms(3, r), init_zero=True)
            assert np.array_equal(y.cpu().numpy(), ref)
    size = it.cache_size()
    it.compile_and_execute("stencil", "float64", list(x.shape), list(x.stride()), None, x.data_ptr(), y.data_ptr(), 0)
    assert it.cache_size() == size and it.cache_hits() >= 1
    assert len(it.last_cache_key()) == 64


def test_interceptor_errors_like_reference():
    b = _basalto()
    it = b._rust.PyBasaltoInterceptor()
    x = torch.zeros(4, 4, 4, 4, device="cuda")
    with pytest.raises(RuntimeError):
        it.compile_and_execute("stencil", "float32", list(x.shape), list(x.stride()), None, x.data_ptr(), x.data_ptr(), 0)
    with pytest.raises(RuntimeError):
        it.compile_and_execute("stencil", "float32", [4, 4], [4], None, 1, 1, 0)
    with pytest.raises(RuntimeError):
        it.compile_and_execute("stencil", "float32", [4, 4], [4, 1], None, 0, 0, 0)
    with pytest.raises(RuntimeError):
        it.compile_and_execute("matmul", "float32", [1, 2, 2, 2], [0, 0, 0, 0], None, 1, 1, 1)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float64])
def test_sweeps_match_iterated_oracle(dtype):
    b = _basalto()
    from basalto import program as P
    for prog, shape, n in ((P.jacobi5_2d(), (130, 256), 7), (P.heat7_3d(), (20, 24, 64), 4),
                           (P.star_3d(P.LAPLACIAN8_COEFFS), (18, 20, 32), 3)):
        x = torch.randn(shape, dtype=dtype, generator=torch.Generator().manual_seed(5))
        a = x.cuda()
        bb = torch.empty_like(a)
        res = b.sweeps(prog, a, bb, n)
        ref = O.sweeps(x.numpy(), lambda u: O.eval_program(u, oracle_terms(prog)), n)
        assert np.array_equal(res.cpu().numpy(), ref)


def test_valid_region_3d_fast_path():
    """The reference's report stencil (7 taps x 0.125 over the valid region) on TMA-friendly sizes."""
    b = _basalto()
    from basalto.program import StencilProgram, Term
    taps = [(1, 1, 1), (0, 1, 1), (2, 1, 1), (1, 0, 1), (1, 2, 1), (1, 1, 0), (1, 1, 2)]
    prog = StencilProgram(3, tuple(Term("mul", 0.125, (t,)) for t in taps), boundary="valid", shrink=(2, 2, 2))
    for shape in ((10, 12, 66), (34, 20, 130), (7, 9, 11)):
        x = torch.randn(shape, generator=torch.Generator().manual_seed(9))
        ref = O.eval_program(x.numpy(), oracle_terms(prog), boundary="valid", shrink=(2, 2, 2))
        assert np.array_equal(b.apply(prog, x.cuda()).cpu().numpy(), ref)


@pytest.mark.parametrize("dtype,shape", [(torch.float32, (257, 300)), (torch.float32, (64, 1024)),
                                         (torch.float32, (3, 124)), (torch.float64, (129, 130)),
                                         (torch.float64, (70, 512)), (torch.float32, (1000, 120))])
def test_temporally_blocked_sweeps_match_oracle(dtype, shape):
    """Multi-sweep 2-D runs fuse several sweeps per launch; every sweep count must give the
    iterated single-sweep result bit for bit, in the buffer the sweeps contract names."""
    b = _basalto()
    from basalto import program as P
    x = torch.rand(shape, dtype=dtype, generator=torch.Generator().manual_seed(17)) * 2 - 1
    prog = P.jacobi5_2d()
    for n in (2, 3, 4, 5, 6, 7, 10, 11, 12, 25):
        a = x.cuda()
        bb = torch.empty_like(a)
        n0 = b.launch_count()
        res = b.sweeps(prog, a, bb, n)
        torch.cuda.synchronize()
        assert (res.data_ptr() == bb.data_ptr()) == (n % 2 == 1)
        ref = O.sweeps(x.numpy(), O.jacobi5_2d, n)
        assert np.array_equal(res.cpu().numpy(), ref), (shape, dtype, n)
        if n >= 3:  # two sweeps cannot fuse and still leave the result in buffer a
            assert b.launch_count() - n0 < n  # sweeps were fused


@pytest.mark.parametrize("shape,fuses", [((37, 61, 132), True), ((20, 28, 120), True), ((9, 5, 8), True),
                                          ((64, 70, 256), True), ((3, 40, 300), True), ((11, 30, 130), False)])
def test_temporally_blocked_3d_heat_matches_oracle(shape, fuses):
    """Multi-sweep 3-D heat runs with max_fused = 2 fuse sweeps per launch (march_tb3d_kernel):
    every sweep count gives the iterated single-sweep result bit for bit.  The shapes cover partial
    tiles in x and y, grids smaller than one tile and than the level warm-up along z, and rows
    and columns that end inside a tile's overlap; rows of 130 floats are not 16-byte aligned,
    so that grid runs single sweeps.  (With pairs of sweeps per launch and the result in the
    buffer the contract names, 2 and 3 sweeps cannot fuse; 4 and more do.)"""
    b = _basalto()
    from basalto import program as P
    x = torch.rand(shape, dtype=torch.float32, generator=torch.Generator().manual_seed(23))
    prog = P.heat7_3d()
    for n in (2, 3, 4, 5, 7, 8):
        a = x.cuda()
        bb = torch.empty_like(a)
        n0 = b.launch_count()
        res = b.sweeps(prog, a, bb, n, max_fused=2)
        torch.cuda.synchronize()
        assert (res.data_ptr() == bb.data_ptr()) == (n % 2 == 1)
        ref = O.sweeps(x.numpy(), O.heat7_3d, n)
        assert np.array_equal(res.cpu().numpy(), ref), (shape, n)
        if n >= 4:
            assert (b.launch_count() - n0 < n) == fuses
