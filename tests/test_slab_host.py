"""Z-slab decomposition logic on CPU ranks (gloo): partition, ghost layout and the exchange
plan, checked by running the oracle on each rank's slab and comparing the gathered grid
with the single-grid oracle — the same layout bst_halo_exchange / bst_slab_sweeps use.
No GPU, no NCCL: ranks are processes exchanging planes with torch.distributed send/recv."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from basalto.slab import SlabLayout, partition
from oracle import stencil_oracle as O


def test_partition_covers_grid():
    for n in (1, 7, 64, 513):
        for p in (1, 2, 3, 8):
            if n < p:
                continue
            spans = [partition(n, p, r) for r in range(p)]
            assert spans[0][0] == 0
            for (s0, c0), (s1, _) in zip(spans, spans[1:]):
                assert s0 + c0 == s1
            assert spans[-1][0] + spans[-1][1] == n
            assert max(c for _, c in spans) - min(c for _, c in spans) <= 1


def test_layout_and_exchange_plan():
    L = SlabLayout((10, 4, 4), 3, 1, 2)
    assert L.n_local == 3 and L.start == 4
    assert L.buffer_shape == (7, 4, 4) and L.owned == slice(2, 5)
    plan = L.exchange_plan()
    assert plan == [(0, slice(2, 4), slice(0, 2)), (2, slice(3, 5), slice(5, 7))]
    assert SlabLayout((10, 4), 1, 0, 1).exchange_plan() == []
    with pytest.raises(ValueError):
        SlabLayout((4, 4, 4), 4, 0, 2).validate()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _exchange(buf: np.ndarray, L: SlabLayout):
    """Ghost exchange by gloo send/recv following SlabLayout.exchange_plan()."""
    reqs = []
    recv = []
    for peer, send_sl, recv_sl in L.exchange_plan():
        t = torch.from_numpy(np.ascontiguousarray(buf[send_sl]))
        reqs.append(dist.isend(t, peer))
        r = torch.empty_like(t)
        reqs.append(dist.irecv(r, peer))
        recv.append((recv_sl, r))
    for q in reqs:
        q.wait()
    for sl, r in recv:
        buf[sl] = r.numpy()


def _worker(rank, world, port, case, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        shape, terms, steps, dtype = case
        g = np.random.default_rng(42)
        x = g.standard_normal(shape).astype(dtype)
        R = max(abs(o[0]) for _, _, taps in terms for o in taps)
        L = SlabLayout(shape, world, rank, R)
        L.validate()
        buf = np.zeros(L.buffer_shape, dtype)
        buf[L.owned] = x[L.start:L.start + L.n_local]
        _exchange(buf, L)
        for _ in range(steps):
            # Same-size sweep over the slab including ghosts; owned planes only read
            # planes within the buffer, beyond the global ends the ghosts stay zero.
            out = O.eval_program(buf, terms)
            nb = np.zeros_like(buf)
            nb[L.owned] = out[L.owned]
            buf = nb
            _exchange(buf, L)
        parts = [None] * world
        dist.all_gather_object(parts, buf[L.owned])
        if rank == 0:
            got = np.concatenate(parts, 0)
            ref = O.sweeps(x, lambda u: O.eval_program(u, terms), steps)
            q.put(bool(np.array_equal(got, ref)))
    finally:
        dist.destroy_process_group()


def _heat_terms():
    return [("mul", 0.4, [(0, 0, 0)]),
            ("mul", 0.1, [(-1, 0, 0), (1, 0, 0), (0, -1, 0), (0, 1, 0), (0, 0, -1), (0, 0, 1)])]


def _star_terms():
    from basalto.program import LAPLACIAN8_COEFFS as c
    t = [("mul", c[0], [(0, 0, 0)])]
    for k in range(1, 5):
        t.append(("mul", c[k], [(k, 0, 0), (-k, 0, 0)]))
        t.append(("mul", c[k], [(0, k, 0), (0, -k, 0)]))
        t.append(("mul", c[k], [(0, 0, k), (0, 0, -k)]))
    return t


@pytest.mark.parametrize("world,case", [
    (2, ((12, 6, 8), _heat_terms(), 3, np.float32)),
    (3, ((13, 5, 7), _heat_terms(), 2, np.float64)),
    (2, ((17, 10, 12), _star_terms(), 2, np.float32)),
    (2, ((9, 16), [("mul", 0.25, [(-1, 0), (1, 0), (0, -1), (0, 1)])], 4, np.float32)),
])
def test_sharded_sweeps_equal_single_grid(world, case):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, case, q)) for r in range(world)]
    for p in procs:
        p.start()
    try:
        ok = q.get(timeout=120)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert ok
    assert all(p.exitcode == 0 for p in procs)


def _deep_worker(rank, world, port, case, q):
    """Deep halos: ghost depth G = k*R, k sweeps per exchange.  Each macro-step evaluates k
    levels over the whole buffer (zeros beyond it), forces levels outside the GLOBAL domain
    to zero (as the fused kernel does with its row range), keeps the owned planes and
    exchanges G planes — the scheme bst_slab_sweeps_deep runs."""
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        shape, terms, steps, k, dtype = case
        g = np.random.default_rng(7)
        x = g.standard_normal(shape).astype(dtype)
        R = max(abs(o[0]) for _, _, taps in terms for o in taps)
        L = SlabLayout(shape, world, rank, k * R)
        L.validate()
        buf = np.zeros(L.buffer_shape, dtype)
        buf[L.owned] = x[L.start:L.start + L.n_local]
        _exchange(buf, L)
        lo_mask = slice(0, L.ghost) if rank == 0 else None
        hi_mask = slice(L.ghost + L.n_local, None) if rank == world - 1 else None
        left = steps
        while left:
            kk = min(k, left)
            cur = buf
            for _ in range(kk):
                cur = O.eval_program(cur, terms)
                for m in (lo_mask, hi_mask):
                    if m is not None:
                        cur[m] = 0
            nb = np.zeros_like(buf)
            nb[L.owned] = cur[L.owned]
            buf = nb
            _exchange(buf, L)
            left -= kk
        parts = [None] * world
        dist.all_gather_object(parts, buf[L.owned])
        if rank == 0:
            got = np.concatenate(parts, 0)
            ref = O.sweeps(x, lambda u: O.eval_program(u, terms), steps)
            q.put(bool(np.array_equal(got, ref)))
    finally:
        dist.destroy_process_group()


_JACOBI = [("mul", 0.25, [(-1, 0), (1, 0), (0, -1), (0, 1)])]


@pytest.mark.parametrize("world,case", [
    (2, ((20, 16), _JACOBI, 7, 3, np.float32)),
    (3, ((31, 12), _JACOBI, 11, 5, np.float32)),
    (3, ((25, 9, 8), _heat_terms(), 5, 2, np.float64)),
])
def test_deep_halo_scheme_equals_single_grid(world, case):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_deep_worker, args=(r, world, port, case, q)) for r in range(world)]
    for p in procs:
        p.start()
    try:
        ok = q.get(timeout=120)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert ok
    assert all(p.exitcode == 0 for p in procs)


def test_slab_ghost_depth_query():
    """bst_slab_ghost_depth (host-only): fused depth k*R for the 2-D Jacobi kernel (k = 4 fp32, 3 fp64), R where
    nothing fuses by default (the 3-D heat kernel fuses only on request, the radius-4 star never); SlabDomain's
    default caps it by the smallest rank's owned planes."""
    from basalto import _abi
    from basalto import program as P
    from basalto.slab import slab_ghost_depth
    assert slab_ghost_depth(P.jacobi5_2d(), (8192, 8192), 1, _abi.BST_F32) == 4
    assert slab_ghost_depth(P.jacobi5_2d(), (8192, 8192), 8, _abi.BST_F64) == 3
    assert slab_ghost_depth(P.jacobi5_2d(), (12, 8192), 4, _abi.BST_F32) == 3
    assert slab_ghost_depth(P.heat7_3d(), (64, 64, 64), 2, _abi.BST_F32) == 1  # 3-D fusion: opt-in only
    assert slab_ghost_depth(P.heat7_3d(), (64, 64, 64), 2, _abi.BST_F64) == 1
    assert slab_ghost_depth(P.heat7_3d().contracted(), (64, 64, 64), 2, _abi.BST_F32) == 1
    assert slab_ghost_depth(P.star_3d(P.LAPLACIAN8_COEFFS), (64, 64, 64), 2, _abi.BST_F32) == 4


def test_fuse_plan_parity():
    from basalto.slab import fuse_plan
    for kmax in (1, 2, 3, 5):
        for n in range(0, 40):
            ks = fuse_plan(n, kmax)
            assert sum(ks) == n and len(ks) % 2 == n % 2 and all(1 <= k <= max(kmax, 1) for k in ks)
    assert fuse_plan(7, 5) == [3, 2, 2] and fuse_plan(10, 5) == [5, 5] and fuse_plan(100, 5) == [5] * 20
    assert fuse_plan(100, 4) == [4] * 22 + [3] * 4 and fuse_plan(2, 4) == [1, 1] and fuse_plan(3, 4) == [3]
    for n in range(4, 60):  # no single-sweep launch once n >= 2 x launches
        ks = fuse_plan(n, 4)
        assert min(ks) >= 2 or n < 2 * len(ks)
