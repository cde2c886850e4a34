"""Z-slab sweeps on GPUs: bst_slab_sweeps / bst_halo_exchange.

* one rank (an NCCL communicator of size 1): the boundary/interior split and the slab
  addressing must give exactly the single-grid result;
* two and four ranks on as many GPUs (skipped with fewer): ghost planes over NCCL, over the
  copy engines, or stored by the sweep kernel itself; gathered result equal to the
  single-grid oracle.  NVLS is off; ranks exchange the NCCL id over gloo; every wait
  is bounded by process-group and join timeouts.
"""
import os
import socket

import numpy as np
import pytest
import torch

from oracle import stencil_oracle as O
from conftest import oracle_terms

pytestmark = pytest.mark.gpu


def _programs():
    from basalto import program as P
    from basalto import workloads as W
    from basalto.program import StencilProgram, Term
    # outside the compiled catalog (runtime-table kernel; its boundary ranges run as two launches)
    odd = StencilProgram(3, (Term("mul", 0.3, ((0, 0, 0), (1, 1, 0))), Term("div", 7.0, ((-1, 0, 2),)),
                             Term("sum", 0.0, ((0, -2, -1), (2, 0, 0)))))
    return [(P.heat7_3d(), (37, 20, 64), torch.float32, 4),
            (P.jacobi5_2d(), (70, 256), torch.float32, 5),
            (P.box(3, 1, W.box27_weights()), (19, 16, 64), torch.float64, 3),
            (P.star_3d(P.LAPLACIAN8_COEFFS), (21, 24, 128), torch.float32, 2),
            (P.jacobi5_2d(), (64, 128), torch.float64, 7),
            (P.jacobi5_2d(), (96, 516), torch.float32, 13),
            (odd, (15, 18, 40), torch.float32, 3)]


@pytest.mark.parametrize("idx", range(7))
def test_single_rank_slab_equals_single_grid(idx):
    from basalto.slab import SlabDomain
    import basalto
    prog, shape, dtype, steps = _programs()[idx]
    x = torch.randn(shape, dtype=dtype, generator=torch.Generator().manual_seed(31))
    dom = SlabDomain(prog, shape, dtype=dtype, device="cuda:0")
    try:
        dom.load(x)
        dom.run(steps)
        got = dom.owned().cpu().numpy()
    finally:
        dom.close()
    a = x.cuda()
    b = torch.empty_like(a)
    ref_gpu = basalto.sweeps(prog, a, b, steps).cpu().numpy()
    ref = O.sweeps(x.numpy(), lambda u: O.eval_program(u, oracle_terms(prog)), steps)
    assert np.array_equal(got, ref_gpu)
    assert np.array_equal(got, ref)


@pytest.mark.parametrize("dtype,shape,steps,ghost", [
    (torch.float32, (70, 256), 7, None),      # default depth 4: plan [3, 2, 2]
    (torch.float32, (64, 520), 10, None),     # [3, 3, 2, 2]
    (torch.float64, (50, 128), 8, None),      # depth 3: [2, 2, 2, 2]
    (torch.float32, (33, 96), 5, 2),          # explicit depth 2: [2, 2, 1]
    (torch.float32, (9, 64), 6, 4),           # owned planes < 2 x depth: boundary launches only
])
def test_single_rank_deep_slab(dtype, shape, steps, ghost):
    """One rank, deep ghosts: fused sweeps over the slab (row range [0, n) as the global
    ends) give exactly the single-grid bits, with one boundary/interior triple of launches
    per fused step."""
    from basalto import program as P
    from basalto.slab import SlabDomain, fuse_plan
    import basalto
    prog = P.jacobi5_2d()
    x = torch.randn(shape, dtype=dtype, generator=torch.Generator().manual_seed(5))
    dom = SlabDomain(prog, shape, dtype=dtype, device="cuda:0", ghost=ghost)
    try:
        G = dom.layout.ghost
        assert G == (ghost if ghost is not None else (4 if dtype == torch.float32 else 3))
        dom.load(x)
        torch.cuda.synchronize()
        n0 = basalto.launch_count()
        dom.run(steps)
        torch.cuda.synchronize()
        launches = basalto.launch_count() - n0
        got = dom.owned().cpu().numpy()
    finally:
        dom.close()
    plan = fuse_plan(steps, G)
    nl = shape[0]
    per = 0
    for k in plan:
        gx = G  # every pass refreshes the full ghost depth
        lo_end = min(gx, nl)
        hi_begin = max(nl - gx, lo_end)
        per += 1 + (hi_begin < nl) + (lo_end < hi_begin)
    assert launches == per
    a = x.cuda()
    ref_gpu = basalto.sweeps(prog, a, torch.empty_like(a), steps).cpu().numpy()
    ref = O.sweeps(x.numpy(), lambda u: O.eval_program(u, oracle_terms(prog)), steps)
    assert np.array_equal(got, ref_gpu)
    assert np.array_equal(got, ref)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _peer_programs():
    """Shapes whose every rank owns at least 2 x radius planes at 4 ranks (peer transport)."""
    from basalto import program as P
    from basalto import workloads as W
    return [(P.heat7_3d(), (37, 20, 64), torch.float32, 4),
            (P.star_3d(P.LAPLACIAN8_COEFFS), (41, 24, 128), torch.float32, 3),
            (P.box(3, 1, W.box27_weights()), (19, 16, 64), torch.float64, 3),
            (P.jacobi5_2d(), (70, 256), torch.float32, 5)]


def _rank(rank, world, port, q, transport="nccl"):
    import datetime

    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        from basalto.slab import SlabDomain
        res = []
        for prog, shape, dtype, steps in (_programs() if transport != "peer" else _peer_programs()):
            x = torch.randn(shape, dtype=dtype, generator=torch.Generator().manual_seed(41))
            dom = SlabDomain(prog, shape, dtype=dtype, device=f"cuda:{rank}", timeout_s=60.0, transport=transport)
            try:
                dom.load(x)
                dom.run(steps)
                torch.cuda.synchronize()
                part = dom.owned().cpu().numpy()
            finally:
                dom.close()
            parts = [None] * world
            dist.all_gather_object(parts, part)
            if rank == 0:
                got = np.concatenate(parts, 0)
                ref = O.sweeps(x.numpy(), lambda u: O.eval_program(u, oracle_terms(prog)), steps)
                res.append(bool(np.array_equal(got, ref)))
        import basalto
        basalto.check_device_errors(rank)  # no bounded wait (TMA stage or neighbour flag) gave up
        if rank == 0:
            q.put(res)
    finally:
        dist.destroy_process_group()


def _spawn(world, transport):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, q, transport)) for r in range(world)]
    for p in procs:
        p.start()
    try:
        res = q.get(timeout=300)
    finally:
        for p in procs:
            p.join(timeout=120)
            if p.is_alive():
                p.kill()
    return res, procs


@pytest.mark.parametrize("world", [2, 4])
def test_ranks_nccl_exchange_equals_single_grid(world):
    """2 ranks: both global ends; 4 ranks: middle ranks with two neighbours as well."""
    if not torch.cuda.is_available() or torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    res, procs = _spawn(world, "nccl")
    assert res == [True] * len(_programs())
    assert all(p.exitcode == 0 for p in procs)


@pytest.mark.parametrize("world", [2, 4])
def test_ranks_copy_engine_transport_equals_single_grid(world):
    """The NCCL path's passes (deep ghosts and fused Jacobi passes included) with the ghost
    planes pushed by the copy engines into the neighbours' mapped buffers and flag-ordered on
    the GPU: the gathered result equals the single-grid oracle bit for bit, and no bounded wait
    for a neighbour's flag expired."""
    if not torch.cuda.is_available() or torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    res, procs = _spawn(world, "copy")
    assert res == [True] * len(_programs())
    assert all(p.exitcode == 0 for p in procs)


@pytest.mark.parametrize("world", [2, 4])
def test_ranks_peer_stores_equal_single_grid(world):
    """Boundary launches store into the neighbours' ghost planes over NVLink (no exchange
    step); the gathered result equals the single-grid oracle bit for bit, and no bounded wait
    for a neighbour's flag expired."""
    if not torch.cuda.is_available() or torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    res, procs = _spawn(world, "peer")
    assert res == [True] * len(_peer_programs())
    assert all(p.exitcode == 0 for p in procs)


def test_single_rank_peer_transport_equals_single_grid():
    """One rank: the peer path (no neighbours) is the boundary/interior split alone."""
    from basalto.slab import SlabDomain
    for prog, shape, dtype, steps in _peer_programs():
        x = torch.randn(shape, dtype=dtype, generator=torch.Generator().manual_seed(8))
        dom = SlabDomain(prog, shape, dtype=dtype, device="cuda:0", transport="peer")
        try:
            dom.load(x)
            dom.run(steps)
            got = dom.owned().cpu().numpy()
        finally:
            dom.close()
        ref = O.sweeps(x.numpy(), lambda u: O.eval_program(u, oracle_terms(prog)), steps)
        assert np.array_equal(got, ref)


@pytest.mark.parametrize("shape,steps", [((40, 33, 132), 5), ((16, 64, 256), 8)])
def test_single_rank_deep_slab_3d_heat(shape, steps):
    """One rank, deep ghosts for the 3-D heat step: fused 3-D sweeps on slabs (row range [0, n)
    as the global ends) give exactly the single-grid bits."""
    from basalto import program as P
    from basalto.slab import SlabDomain
    prog = P.heat7_3d()
    x = torch.rand(shape, generator=torch.Generator().manual_seed(3))
    dom = SlabDomain(prog, shape, device="cuda:0", ghost=2)  # deeper ghosts than the default: fused pairs
    try:
        assert dom.layout.ghost == 2
        dom.load(x)
        dom.run(steps)
        got = dom.owned().cpu().numpy()
    finally:
        dom.close()
    ref = O.sweeps(x.numpy(), lambda u: O.eval_program(u, oracle_terms(prog)), steps)
    assert np.array_equal(got, ref)
