"""Z-slab domain decomposition across GPUs (one process per GPU).

The reference's only parallelism is spatial decomposition with halo exchange
(crates/basalto-communication/src/halo_exchange.rs): every rank owns a sub-grid and trades
boundary slabs with rank±1 over NCCL (or MPI through host memory), periodically, and the
received slab overwrites owned boundary data (halo_exchange.rs:111-164).  Here axis 0 of
a 2-D/3-D grid is split into contiguous slabs; each rank stores its slab with `ghost`
extra planes on either side:

    buffer[0 : g]            lower ghost  (rank-1's last g owned planes; zeros on rank 0)
    buffer[g : g + n_local]  owned planes
    buffer[g+n_local : ...]  upper ghost  (rank+1's first g owned planes; zeros on the last rank)

Global ends are Dirichlet-0 (not periodic), so the sharded result equals the single-grid
result point for point.  The exchange is one NCCL group of contiguous send/recv pairs (no
packing), issued by the C library on its own stream and overlapped with the interior
sweep (bst_slab_sweeps_deep).  Plumbing (ranks, the NCCL unique id) goes through
torch.distributed.

Deep halos: where a kernel fuses k sweeps per pass (temporal blocking), the ghost depth is
k x radius and the slab exchanges once per k sweeps instead of once per sweep; the depth
defaults to what the library reports for the program (bst_slab_ghost_depth), capped by the
smallest rank's owned planes.

Copy transport (transport="copy", bst_slab_sweeps_copy): the same passes as the NCCL path,
with the ghost planes pushed by the copy engines over NVLink (cudaMemcpyAsync into CUDA IPC
peer mappings of the neighbours' buffers) and a sequence flag raised in the neighbours'
memory; the boundary rows of the next pass wait (bounded, on the GPU) for those flags.  The
copies take no SMs, so they overlap an interior launch that holds all of them.

Peer transport (transport="peer", bst_slab_sweeps_p2p): no exchange step at all.  Every
sweep is one kernel launch whose boundary work items copy their output planes, through the
peer mappings, straight into the neighbours' ghost planes, then raise a sequence flag in the
neighbour's memory; items that read ghost planes wait (bounded) for the neighbours' previous
sweep.

With the copy and peer transports the neighbours write into this rank's buffers
asynchronously: load() belongs before the first run().
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from . import _abi
from .program import StencilProgram


def partition(n: int, nranks: int, rank: int) -> tuple[int, int]:
    """(first owned plane, number of owned planes): balanced, the remainder to low ranks."""
    if not 0 <= rank < nranks:
        raise ValueError("rank out of range")
    base, rem = divmod(n, nranks)
    count = base + (1 if rank < rem else 0)
    start = rank * base + min(rank, rem)
    return start, count


@dataclass(frozen=True)
class SlabLayout:
    global_shape: tuple[int, ...]
    nranks: int
    rank: int
    ghost: int

    @property
    def start(self) -> int:
        return partition(self.global_shape[0], self.nranks, self.rank)[0]

    @property
    def n_local(self) -> int:
        return partition(self.global_shape[0], self.nranks, self.rank)[1]

    @property
    def local_shape(self) -> tuple[int, ...]:
        return (self.n_local,) + tuple(self.global_shape[1:])

    @property
    def buffer_shape(self) -> tuple[int, ...]:
        return (self.n_local + 2 * self.ghost,) + tuple(self.global_shape[1:])

    @property
    def owned(self) -> slice:
        """Owned planes inside the buffer."""
        return slice(self.ghost, self.ghost + self.n_local)

    @property
    def plane_elems(self) -> int:
        n = 1
        for s in self.global_shape[1:]:
            n *= s
        return n

    def neighbours(self) -> tuple[int | None, int | None]:
        lo = self.rank - 1 if self.rank > 0 else None
        hi = self.rank + 1 if self.rank < self.nranks - 1 else None
        return lo, hi

    def exchange_plan(self):
        """[(peer, send_slice, recv_slice)] in buffer coordinates — the contiguous plane
        ranges bst_halo_exchange moves (sends the first/last `ghost` owned planes)."""
        g, n = self.ghost, self.n_local
        lo, hi = self.neighbours()
        plan = []
        if g == 0:
            return plan
        if lo is not None:
            plan.append((lo, slice(g, 2 * g), slice(0, g)))
        if hi is not None:
            plan.append((hi, slice(n, n + g), slice(n + g, n + 2 * g)))
        return plan

    def validate(self):
        if self.n_local < max(self.ghost, 1):
            raise ValueError(f"rank {self.rank} owns {self.n_local} planes; needs at least "
                             f"{max(self.ghost, 1)} for a radius-{self.ghost} stencil")


def fuse_plan(nsteps: int, kmax: int) -> list[int]:
    """Sweeps per fused launch for nsteps ping-pong sweeps, as the C library plans them: the
    fewest launches of at most kmax sweeps, one more if their count does not have nsteps'
    parity (the result then lands in the buffer a per-sweep ping-pong would use), with the
    sweeps spread evenly over them, larger launches first."""
    if kmax < 2 or nsteps < 2:
        return [1] * max(nsteps, 0)
    launches = -(-nsteps // kmax)
    if launches % 2 != nsteps % 2:
        launches += 1
    base, rem = divmod(nsteps, launches)
    return [base + (1 if i < rem else 0) for i in range(launches)]


def slab_ghost_depth(program: StencilProgram, global_shape, nranks: int, dtype_code: int) -> int:
    """Ghost planes per side for a slab run: the library's fused-sweep depth for this program
    (a multiple of the axis-0 radius), capped by the smallest rank's owned planes.  Every rank
    computes the same value from the same arguments."""
    r = program.radius()[0]
    smallest = min(partition(global_shape[0], nranks, k)[1] for k in range(nranks))
    local = (smallest,) + tuple(global_shape[1:])
    depth = ctypes.c_int32(0)
    cprog = program.to_c(local)
    _abi.check(_abi.lib().bst_slab_ghost_depth(ctypes.byref(cprog), dtype_code, len(local), _abi.i64_array(local),
                                               ctypes.byref(depth)))
    g = int(depth.value)
    if nranks > 1 and r > 0 and g > smallest:
        g = max(r, smallest // r * r)
    return max(g, r)


class SlabDomain:
    """A sharded grid on this rank's GPU with a ghost-exchanging sweep loop.

    Create it after torch.distributed is initialised (any backend; it only broadcasts the
    NCCL unique id).  `load(global_grid_or_local)` fills the owned planes; `run(n)` performs
    n overlapped sweeps; `gather()` returns the global grid on every rank (for tests).
    """

    def __init__(self, program: StencilProgram, global_shape, dtype=torch.float32, device=None,
                 timeout_s: float = 120.0, group=None, ghost: int | None = None, transport: str = "nccl"):
        import torch.distributed as dist

        if transport not in ("nccl", "copy", "peer"):
            raise ValueError("transport is 'nccl' (exchange over NCCL), 'copy' (copy engines over NVLink) or "
                             "'peer' (boundary stores over NVLink)")
        self.transport = transport
        if program.boundary != "zero" or program.ndim not in (2, 3) or program.ndim != len(global_shape):
            raise ValueError("slab sweeps need a same-size 2-D or 3-D program")
        self.program = program
        self.dtype = dtype
        ws = dist.get_world_size(group) if dist.is_initialized() else 1
        rank = dist.get_rank(group) if dist.is_initialized() else 0
        gshape = tuple(int(s) for s in global_shape)
        self._dt = _abi.BST_F32 if dtype == torch.float32 else _abi.BST_F64
        if ghost is None:
            # peer transport sweeps one step per pass: ghosts as deep as the axis-0 radius
            ghost = slab_ghost_depth(program, gshape, ws, self._dt) if transport != "peer" else program.radius()[0]
        self.layout = SlabLayout(gshape, ws, rank, int(ghost))
        if self.layout.ghost < program.radius()[0]:
            raise ValueError("ghost depth is below the program's axis-0 radius")
        self.layout.validate()
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        self.a = torch.zeros(self.layout.buffer_shape, dtype=dtype, device=self.device)
        self.b = torch.zeros_like(self.a)
        self._cprog = program.to_c(self.layout.local_shape)
        obj = [None]
        if rank == 0:
            uid = (ctypes.c_uint8 * 128)()
            _abi.check(_abi.lib().bst_nccl_get_unique_id(uid))
            obj[0] = bytes(uid)
        if ws > 1:
            dist.broadcast_object_list(obj, src=0, group=group)
        uid = (ctypes.c_uint8 * 128).from_buffer_copy(obj[0])
        h = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            _abi.check(_abi.lib().bst_comm_create(uid, ws, rank, self.device.index, float(timeout_s), ctypes.byref(h)))
        self._comm = h
        self.current = self.a
        if transport != "nccl":  # collective: every rank registers its two buffers in this order
            for buf in (self.a, self.b):
                with torch.cuda.device(self.device):
                    _abi.check(_abi.lib().bst_comm_register_slab(self._comm, ctypes.c_void_p(buf.data_ptr()), self._dt,
                                                                 self.layout.plane_elems, self.layout.n_local,
                                                                 self.layout.ghost))

    def _stream(self):
        return ctypes.c_void_p(torch.cuda.current_stream(self.device).cuda_stream)

    def load(self, grid: torch.Tensor):
        """Fill owned planes from the global grid (or this rank's local slab) and exchange ghosts."""
        L = self.layout
        src = grid[L.start:L.start + L.n_local] if tuple(grid.shape) == L.global_shape else grid
        self.a.zero_()
        self.b.zero_()
        self.a[L.owned].copy_(src.to(self.device, self.dtype))
        self.current = self.a
        self.exchange(self.a)

    def exchange(self, buf: torch.Tensor):
        L = self.layout
        with torch.cuda.device(self.device):
            _abi.check(_abi.lib().bst_halo_exchange(self._comm, ctypes.c_void_p(buf.data_ptr()), self._dt,
                                                    L.plane_elems, L.n_local, L.ghost, self._stream()))

    def run(self, nsteps: int) -> torch.Tensor:
        """nsteps sweeps; returns the buffer holding the result (ghosts valid)."""
        L = self.layout
        other = self.b if self.current is self.a else self.a
        fn = {"nccl": _abi.lib().bst_slab_sweeps_deep, "copy": _abi.lib().bst_slab_sweeps_copy,
              "peer": _abi.lib().bst_slab_sweeps_p2p}[self.transport]
        with torch.cuda.device(self.device):
            _abi.check(fn(
                self._comm, ctypes.byref(self._cprog), self._dt, len(L.local_shape), _abi.i64_array(L.local_shape),
                L.ghost, ctypes.c_void_p(self.current.data_ptr()), ctypes.c_void_p(other.data_ptr()), int(nsteps),
                self._stream()))
        if nsteps % 2:
            self.current = other
        return self.current

    def owned(self) -> torch.Tensor:
        return self.current[self.layout.owned]

    def gather(self) -> torch.Tensor:
        """The global grid assembled on every rank (all_gather of owned slabs)."""
        import torch.distributed as dist

        L = self.layout
        if L.nranks == 1:
            return self.owned().clone()
        mine = self.owned().contiguous()
        sizes = [partition(L.global_shape[0], L.nranks, r)[1] for r in range(L.nranks)]
        bufs = [torch.empty((s,) + L.global_shape[1:], dtype=self.dtype, device=self.device) for s in sizes]
        dist.all_gather(bufs, mine)
        return torch.cat(bufs, 0)

    def close(self):
        if self._comm:
            torch.cuda.synchronize(self.device)
            _abi.lib().bst_comm_destroy(self._comm)
            self._comm = None

    def abort(self):
        if self._comm:
            _abi.lib().bst_comm_abort(self._comm)
            self._comm = None

    def __del__(self):  # pragma: no cover - best effort
        try:
            self.close()
        except Exception:
            pass
