"""Benchmark of the stencil hot path (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl basalto|reference] [--workload NAME]
    torchrun --nproc-per-node N bench.py --gpus N ...       (N > 1: one process per GPU)

Workload (default): the 25-point 8th-order star (radius 4), fp32 1024 x 1024 x 1024 ~N(0,1)
seed 4, Dirichlet-0 ghost cells, 10 sweeps.  One step = the 10 sweeps applied to the seeded
grid, which stays unchanged (sweep 1 reads it, sweeps 2..10 ping-pong two more buffers), so
every step does the same work and its result can be checked.  The grid is the largest
single-GPU configuration (1.07 G points, 4 GiB).

N > 1: the grid is split along Z into one slab per GPU.  "strong" workloads (star-25,
heat-7) split the one global grid; "weak" ones (box-27 768^3, the 2-D Jacobi grid) stack one
grid per GPU.  Every rank generates the same seeded global grid on its GPU and keeps its slab
plus ghost planes, so the N-GPU result is the single-grid result point for point.  Per sweep
the boundary planes are computed first, their ghost planes cross NVLink in one NCCL group on
a side stream, and the interior planes compute meanwhile (bst_slab_sweeps_deep).

value      grid-point updates per second of the whole job (Gpts/s), inputs resident in HBM,
           CUDA events on the compute stream, max over ranks.  Inputs smaller than L2 are
           timed step by step with a 256 MiB write between steps.
parity     after the timed steps, sampled output points (global ends, every rank's first and
           last planes, random points) are recomputed by the CPU oracle from their input
           neighbourhood and compared bit for bit; summed over ranks.
e2e        the same metric through the public API with host buffers: every step copies the
           seeded grid in from pinned host memory, runs the sweeps (basalto.apply +
           basalto.sweeps, the C ABI's bst_stencil_apply + bst_stencil_sweeps; at N > 1
           bst_halo_exchange + bst_slab_sweeps_deep per rank) and copies the result back, three
           buffer sets in flight, uploads and downloads on separate copy streams.
           e2e.torch_compile_per_sweep: torch.compile(fn, backend="basalto") called once per
           sweep (the drop-in plugin path), N = 1.
roofline   the dominant kernel: algorithmic bytes (2 x element size per point: one read + one
           write) per pass over this rank's grid / average pass time, against the measured HBM
           copy bandwidth; a temporally blocked pass performs several sweeps for those bytes.
passes     (N > 1) per-pass device times of the boundary launches, the ghost exchange and the
           interior launch (CUDA events, two extra untimed steps, max over ranks).
halo       (N > 1) ghost planes, bytes and time of one exchange timed alone.
energy     NVML total-energy counter over at least one second of steps, summed over ranks.
cpu_baseline / --impl reference
           the reference's CPU path: eager torch through the reference backend's control
           flow (oracle/reference_path.py), all host threads, on a bounded Z-slab sample of the
           seeded grid.  The reference arm loads none of this repository's native libraries.
--contract fused multiply-add arithmetic (BST_PROGRAM_CONTRACT); --dtype / --shape override
           the workload's element type / grid.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
PKG_DIR = REPO / "bs-compiler_b200" / "basalto"
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))

import numpy as np  # noqa: E402
import torch  # noqa: E402

METRIC = "stencil Gpts/s and % of HBM roofline at 1/2/4/8 B200 vs reference CPU path"
UNIT = "Gpts/s"
FALLBACK_HBM_GBS = 6650.0
DEFAULT_WORKLOAD = "star25_3d"


def _peaks():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            d = json.loads(p.read_text())
            return float(d["hbm_gbs"]), "measured"
        except Exception:
            pass
    return FALLBACK_HBM_GBS, "fallback"


def _traffic(workload: str, kernel: str):
    """Per-launch DRAM bytes of the kernel from a committed ncu summary, if one exists."""
    p = REPO / "profiles" / "traffic.json"
    if not p.exists():
        return None
    try:
        d = json.loads(p.read_text())
        return d.get(workload, {}).get(kernel)
    except Exception:
        return None


# ---- workload definitions ------------------------------------------------------------------

def _workload_table(native: bool):
    """The workload table.  native: through the `basalto` package (which loads the native
    library).  Otherwise program.py and workloads.py are loaded as a stand-alone package
    without the package's __init__, so no native library of this repository is mapped (the
    reference arm times the reference's CPU path alone)."""
    if native:
        if str(PKG_DIR.parent) not in sys.path:
            sys.path.insert(0, str(PKG_DIR.parent))
        from basalto.workloads import WORKLOADS
        return WORKLOADS
    import importlib
    import types
    name = "_basalto_definitions"
    if name not in sys.modules:
        pkg = types.ModuleType(name)
        pkg.__path__ = [str(PKG_DIR)]
        sys.modules[name] = pkg
    return importlib.import_module(f"{name}.workloads").WORKLOADS


def _workload(args, table):
    """The named workload, optionally on a different grid / dtype / arithmetic."""
    import dataclasses
    w = table[args.workload]
    if args.shape:
        w = dataclasses.replace(w, shape=tuple(int(v) for v in args.shape.split("x")))
    if args.dtype:
        w = dataclasses.replace(w, dtype={"f32": torch.float32, "f64": torch.float64}[args.dtype])
    if args.contract:  # fused multiply-add folding (the reference GPU kernel's arithmetic)
        w = dataclasses.replace(w, program=w.program.contracted())
        os.environ["BASALTO_FP_CONTRACT"] = "1"  # the torch.compile leg compiles the same program
    return w


def _dtype_name(w):
    return "f32" if w.dtype == torch.float32 else "f64"


def _native_maps():
    """This repository's native libraries mapped into the process (Linux /proc/self/maps)."""
    try:
        lines = Path("/proc/self/maps").read_text().splitlines()
    except OSError:
        return []
    hits = set()
    for ln in lines:
        f = ln.split()
        if f and f[-1].startswith(str(REPO)) and f[-1].endswith(".so"):
            hits.add(f[-1])
    return sorted(hits)


def cpu_sample_shape(w):
    """The bounded sample the CPU legs sweep: a Z-slab of at most 64 planes of a 3-D grid, at
    most 2048 rows of a 2-D grid, the whole 1-D grid."""
    if len(w.shape) == 3:
        return (min(w.shape[0], 64),) + tuple(w.shape[1:])
    if len(w.shape) == 2:
        return (min(w.shape[0], 2048), w.shape[1])
    return tuple(w.shape)


# ---- device-side helpers ---------------------------------------------------------------------

class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 50 ms during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines = []
        self.t = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "50"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if not self.proc:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.t.join(timeout=2)
        sm, pw, mx, reasons = [], [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
                pw.append(float(f[3]))
            except ValueError:
                continue
            for name, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(name)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm),
                "power_w_median": statistics.median(pw) if pw else None}


class EnergyMeter:
    """NVML total-energy counter (millijoules since driver load)."""

    def __init__(self, index: int):
        self.nv = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.nv = pynvml
        except Exception:
            self.nv = None

    def read(self):
        if self.nv is None:
            return None
        try:
            return float(self.nv.nvmlDeviceGetTotalEnergyConsumption(self.h))
        except Exception:
            return None


E2E_SETS = 3  # device buffer sets of the end-to-end pipeline

TRANSPORT_NOTE = {
    "nccl": "NCCL ghost exchange on a side stream, overlapped with the interior",
    "copy": "ghost planes pushed by the copy engines over NVLink, overlapped with the interior",
    "peer": "boundary planes stored into the neighbours over NVLink by the sweep kernel",
}


def pipelined(n_steps, upload, compute, download, stream, nsets=E2E_SETS):
    """Time n_steps end-to-end steps with nsets buffer sets in flight.

    Step k uses set k % nsets: its host->device upload runs on one copy stream, its compute on
    `stream`, its device->host download on a second copy stream (PCIe is full duplex).  With
    three sets the upload of step k+1 and the download of step k-1 overlap each other and step
    k's compute, and an upload never waits for the download just before it.  Every step still
    copies its own input in and its own result out inside the timed region.  upload(s),
    compute(s) and download(s) enqueue on the current stream.  Returns ms per step (CUDA
    events on `stream`)."""
    h2d, d2h = torch.cuda.Stream(), torch.cuda.Stream()
    ev_in = [torch.cuda.Event() for _ in range(nsets)]
    ev_done = [torch.cuda.Event() for _ in range(nsets)]
    ev_free = [None] * nsets

    def run(n):
        for k in range(n):
            s = k % nsets
            with torch.cuda.stream(h2d):
                if ev_free[s] is not None:
                    h2d.wait_event(ev_free[s])
                upload(s)
                ev_in[s].record(h2d)
            with torch.cuda.stream(stream):
                stream.wait_event(ev_in[s])
                compute(s)
                ev_done[s].record(stream)
            with torch.cuda.stream(d2h):
                d2h.wait_event(ev_done[s])
                download(s)
                ev_free[s] = torch.cuda.Event()
                ev_free[s].record(d2h)
        for e in ev_free:
            if e is not None:
                stream.wait_event(e)

    run(nsets)  # warm-up
    torch.cuda.synchronize()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record(stream)
    h2d.wait_event(f0)
    run(n_steps)
    f1.record(stream)
    torch.cuda.synchronize()
    return f0.elapsed_time(f1) / n_steps


def _dist():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def _init_pg(ws, rank, local, backend):
    import datetime

    import torch.distributed as dist
    if ws > 1 and not dist.is_initialized():
        dist.init_process_group(backend, rank=rank, world_size=ws, timeout=datetime.timedelta(seconds=180),
                                device_id=torch.device("cuda", local) if backend == "nccl" else None)
    return dist


# ---- CPU legs ------------------------------------------------------------------------------

class CpuReference:
    """Eager torch on the host through the reference backend's control flow, on a bounded
    sample grid of the workload (cpu_sample_shape), every sweep from the seeded sample."""

    def __init__(self, workload, threads: int | None = None):
        from oracle.reference_path import compile_reference
        if threads:
            torch.set_num_threads(threads)
        self.w = workload
        self.shape = cpu_sample_shape(workload)
        self.x = workload.make_input(shape=self.shape)  # CPU generator: the configuration's seeded stream
        self.points = int(np.prod(self.shape))
        self.cf = compile_reference(workload.fn)
        self.cf(self.x)  # compile + one warm sweep

    def sweep(self):
        t0 = time.perf_counter()
        self.cf(self.x)
        return time.perf_counter() - t0

    def rate_for(self, seconds: float):
        """(Gpts/s, seconds, sweeps): whole sweeps until `seconds` of host work have run."""
        n, dt = 0, 0.0
        while dt < seconds:
            dt += self.sweep()
            n += 1
        return self.points * n / dt / 1e9, dt, n

    def describe(self):
        return (f"one sweep per step over a {'x'.join(map(str, self.shape))} sample of the "
                f"{'x'.join(map(str, self.w.shape))} grid (same distribution and seed), eager torch through the "
                f"reference backend's control flow")


def run_reference(args):
    ws, rank, local = _dist()
    if rank != 0:
        return
    table = _workload_table(native=False)
    w = _workload(args, table)
    threads = os.cpu_count() or 1
    ref = CpuReference(w, threads)
    times = []
    for i in range(args.warmup + args.steps):
        dt = ref.sweep()
        if i >= args.warmup:
            times.append(dt)
    ms = statistics.median(times) * 1e3
    value = ref.points / (ms * 1e-3) / 1e9
    loaded = _native_maps()
    line = {
        "metric": METRIC, "value": round(value, 4), "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 3), "higher_is_better": True,
        "scaling": w.scaling if w.scaling != "replicas" else "weak", "vs_baseline": None,
        "dtype": _dtype_name(w), "data": "synthetic", "impl": "reference",
        "config": {"workload": w.label(), "sample": ref.describe(),
                   "step": "one sampled sweep (ms_per_step is the time of that sweep)"},
        "cpu_baseline": {"value": round(value, 4), "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": ref.describe()},
        "e2e": {"value": round(value, 4), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "native_libraries_loaded": loaded,
    }
    if loaded:
        raise SystemExit(f"reference arm mapped this repository's native code: {loaded}")
    print(json.dumps(line), flush=True)


# ---- parity: sampled points against the oracle ---------------------------------------------

def sample_points(gshape, owners, seed=11, n_random=4):
    """Global output points to check: grid corners, every rank's first and last two planes,
    plus random points.  owners: list of (start, n_local) per rank along axis 0."""
    g = np.random.default_rng(seed)
    nd = len(gshape)
    zs = {0, gshape[0] - 1}
    for s, n in owners:
        for z in (s, s + 1, s + n - 2, s + n - 1):
            if 0 <= z < gshape[0]:
                zs.add(z)
    pts = []
    for i, z in enumerate(sorted(zs)):
        rest = [int(g.integers(0, e)) if (i % 3) else (0 if i % 2 else e - 1) for e in gshape[1:]]
        pts.append([z] + rest)
    for _ in range(n_random):
        pts.append([int(g.integers(0, e)) for e in gshape])
    if nd == 3:
        pts.append([gshape[0] - 1, gshape[1] - 1, 0])
    return [tuple(p) for p in pts]


def oracle_at_point(x_box: np.ndarray, box_lo, gshape, point, prog, sweeps: int):
    """The program's value after `sweeps` sweeps at global `point`, computed by the oracle from
    the input box x_box (global origin box_lo) covering point +- sweeps x radius, clipped to
    the grid.  After every sweep the box loses `radius` cells on each face that is not a grid
    face (their zero padding is not the real neighbourhood), so what remains is exact."""
    from oracle import stencil_oracle as O
    terms = [(t.op, t.scale, t.taps) for t in prog.terms]
    R = prog.radius()
    x = x_box
    lo = list(box_lo)
    for _ in range(sweeps):
        x = O.eval_program(x, terms, prog.init_zero, "zero")
        sl = []
        for a in range(x.ndim):
            c0 = R[a] if lo[a] > 0 else 0
            c1 = R[a] if lo[a] + x.shape[a] < gshape[a] else 0
            sl.append(slice(c0, x.shape[a] - c1))
            lo[a] += c0
        x = x[tuple(sl)]
    return x[tuple(point[a] - lo[a] for a in range(x.ndim))]


def neighbourhood(x_global: torch.Tensor, point, reach):
    lo = [max(0, p - r) for p, r in zip(point, reach)]
    hi = [min(e, p + r + 1) for p, r, e in zip(point, reach, x_global.shape)]
    box = x_global[tuple(slice(a, b) for a, b in zip(lo, hi))].cpu().numpy()
    return box, lo


# ---- the measured arm ----------------------------------------------------------------------

def run_basalto(args):
    if str(PKG_DIR.parent) not in sys.path:
        sys.path.insert(0, str(PKG_DIR.parent))
    import basalto
    from basalto import _abi
    from basalto.slab import fuse_plan, partition, slab_ghost_depth

    ws, rank, local = _dist()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = _init_pg(ws, rank, local, "nccl") if ws > 1 else None
    w = _workload(args, _workload_table(native=True))
    prog = w.program
    sweeps = w.steps
    stream = torch.cuda.current_stream(dev)
    es = w.elem_size
    lib = _abi.lib()
    dt = _abi.BST_F32 if w.dtype == torch.float32 else _abi.BST_F64
    sp = ctypes.c_void_p(stream.cuda_stream)
    sharded = ws > 1 and w.scaling in ("strong", "weak")
    gshape = w.global_shape(ws) if sharded else tuple(w.shape)

    # The seeded global grid, generated on this GPU (every rank generates the same grid).
    x_global = w.make_input(shape=gshape, device=dev)
    R = prog.radius()
    reach = [r * sweeps for r in R]

    comm = None
    if not sharded:
        owners = [(0, gshape[0])]
        my_start, n_local = 0, gshape[0]
        x0 = x_global
        if prog.boundary == "zero":
            a = torch.empty_like(x0)
            b = torch.empty_like(x0)

            def step_on(src, pa, pb):
                basalto.apply(prog, src, out=pa)
                return basalto.sweeps(prog, pa, pb, sweeps - 1) if sweeps > 1 else pa

            def step():
                return step_on(x0, a, b)
        else:  # a shrinking (valid-region) stencil: every sweep from the input into its own output
            b = torch.empty(prog.out_shape(x0.shape), dtype=x0.dtype, device=dev)

            def step_on(src, pa, pb):
                for _ in range(sweeps):
                    basalto.apply(prog, src, out=pb)
                return pb

            def step():
                return step_on(x0, None, b)
        local_points = w.points
        points_job = w.points * (ws if ws > 1 else 1)  # replicas: every rank runs the whole grid
        if ws > 1:
            owners = [(0, gshape[0])]
    else:
        owners = [partition(gshape[0], ws, r) for r in range(ws)]
        my_start, n_local = owners[rank]
        transport = args.transport
        if transport == "auto":
            # Measured on B200: at 2 GPUs the NCCL path (boundary launches concurrent with the
            # interior) leads; from 4 GPUs on the copy engines match or beat it, since NCCL's
            # kernel and the boundary launches then wait for SMs the interior launch holds.
            transport = "nccl" if ws <= 2 else "copy"
        G = slab_ghost_depth(prog, gshape, ws, dt) if transport != "peer" else R[0]
        if args.ghost:
            smallest = min(o[1] for o in owners)
            if transport == "peer" or R[0] == 0 or args.ghost % R[0] or not R[0] <= args.ghost <= smallest:
                raise SystemExit(f"--ghost {args.ghost}: the NCCL and copy transports take a multiple of the axis-0 radius "
                                 f"({R[0]}) up to the smallest slab ({smallest} planes)")
            G = args.ghost
        local_shape = [n_local] + list(gshape[1:])
        plane = int(np.prod(gshape[1:]))
        x0 = torch.zeros([n_local + 2 * G] + list(gshape[1:]), dtype=w.dtype, device=dev)
        lo, hi = max(0, my_start - G), min(gshape[0], my_start + n_local + G)
        x0[lo - (my_start - G):hi - (my_start - G)].copy_(x_global[lo:hi])
        a = torch.zeros_like(x0)
        b = torch.zeros_like(x0)
        uid = (ctypes.c_uint8 * 128)()
        obj = [None]
        if rank == 0:
            _abi.check(lib.bst_nccl_get_unique_id(uid))
            obj[0] = bytes(uid)
        dist.broadcast_object_list(obj, src=0)
        uid = (ctypes.c_uint8 * 128).from_buffer_copy(obj[0])
        h = ctypes.c_void_p()
        _abi.check(lib.bst_comm_create(uid, ws, rank, local, 120.0, ctypes.byref(h)))
        comm = h
        cp = prog.to_c(local_shape)
        shp = _abi.i64_array(local_shape)
        sweep_fn = {"nccl": lib.bst_slab_sweeps_deep, "copy": lib.bst_slab_sweeps_copy,
                    "peer": lib.bst_slab_sweeps_p2p}[transport]

        def register(buf):  # collective: every rank registers its buffers in the same order
            if transport != "nccl":
                _abi.check(lib.bst_comm_register_slab(comm, ctypes.c_void_p(buf.data_ptr()), dt, plane, n_local, G))

        register(a)
        register(b)

        def slab_sweeps(src, dst, n):
            _abi.check(sweep_fn(comm, ctypes.byref(cp), dt, len(local_shape), shp, G,
                                ctypes.c_void_p(src.data_ptr()), ctypes.c_void_p(dst.data_ptr()), n, sp))

        def step_on(src, pa, pb):
            slab_sweeps(src, pa, 1)          # sweep 1 reads the seeded slab, which stays unchanged
            if sweeps > 1:
                slab_sweeps(pa, pb, sweeps - 1)
                return pb if (sweeps - 1) % 2 else pa
            return pa

        def step():
            return step_on(x0, a, b)

        kmax = max(1, G // R[0]) if R[0] and transport != "peer" else 1
        slab_passes = 1 + len(fuse_plan(sweeps - 1, kmax))
        local_points = n_local * plane
        points_job = int(np.prod(gshape))

    # Parity sample: the input neighbourhood of every sampled point this rank owns.
    check = []
    if prog.boundary == "zero":
        for p in sample_points(gshape, owners):
            if my_start <= p[0] < my_start + n_local or not sharded:
                box, lo_box = neighbourhood(x_global, p, reach)
                check.append((p, box, lo_box))
    else:
        pts = [(0,), (w.out_points - 1,), (w.out_points // 2,)]
        for p in pts:
            check.append((p, x_global[p[0]:p[0] + 3].cpu().numpy(), None))
    if sharded:
        del x_global
        torch.cuda.empty_cache()

    # ---- timed region (device time, CUDA events on the compute stream) -------------------
    l2_bytes = 126 << 20
    flush = None
    if local_points * es < l2_bytes:  # the input fits in L2: flush it between timed steps
        flush = torch.zeros(256 << 20, dtype=torch.uint8, device=dev)
        l2_note = "L2 flushed before every timed step (256 MiB write, outside the timed windows)"
    else:
        l2_note = f"inputs larger than L2 ({local_points * es / 2**20:.0f} MiB grid per GPU, 3 buffers)"
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    clocks = ClockSampler(local)
    clocks.start()
    n0 = basalto.launch_count()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    result = None
    if flush is None:  # inputs larger than L2: consecutive steps cannot hit in L2
        e0.record(stream)
        for _ in range(args.steps):
            result = step()
        e1.record(stream)
        torch.cuda.synchronize()
        ms_total = e0.elapsed_time(e1)
    else:  # small inputs: L2 flushed before every step, each step timed on its own
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
        for a0, a1 in evs:
            flush.add_(1)  # writes 256 MiB (> L2) between timed steps
            a0.record(stream)
            result = step()
            a1.record(stream)
        torch.cuda.synchronize()
        ms_total = sum(a0.elapsed_time(a1) for a0, a1 in evs)
    if dist:
        dist.barrier()
    launches = basalto.launch_count() - n0
    clk = clocks.stop()
    if dist:
        t = torch.tensor([ms_total], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_total = float(t.item())
    ms_step = ms_total / args.steps
    value = points_job * sweeps * args.steps / (ms_total * 1e-3) / 1e9

    # ---- parity of the last timed step's result ----------------------------------------------
    basalto.check_device_errors(local)
    bad, checked = 0, 0
    for p, box, lo_box in check:
        if prog.boundary == "zero":
            want = oracle_at_point(box, lo_box, gshape, p, prog, sweeps)
            if sharded:
                got = result[(p[0] - my_start + G,) + tuple(p[1:])].item()
            else:
                got = result[p].item()
        else:
            from oracle import stencil_oracle as O
            want = O.eval_program(box, [(t.op, t.scale, t.taps) for t in prog.terms], prog.init_zero, "valid",
                                  prog.shrink)[0]
            got = result[p].item()
        checked += 1
        if not (np.array_equal(np.asarray(want), np.asarray(got, dtype=box.dtype))):
            bad += 1
    if dist:
        t = torch.tensor([bad, checked], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        bad, checked = int(t[0].item()), int(t[1].item())
    parity = {"ok": bad == 0 and checked > 0, "points": checked, "mismatches": bad,
              "against": "CPU oracle (oracle/stencil_oracle.py) folded over each point's input neighbourhood, "
                         "bit for bit, after the last timed step"}

    # ---- energy over at least one second of steps ----------------------------------------
    energy = None
    meter = EnergyMeter(local)
    if True:  # every rank runs these steps (they exchange ghosts), whether or not its NVML answers
        if dist:
            dist.barrier()
        torch.cuda.synchronize()
        # The same number of steps on every rank (their sweeps exchange with each other): at least
        # a second's worth by the timed steps' duration, which is already the max over ranks.
        n_energy = max(args.steps, int(1000.0 / max(ms_step, 1e-3)) + 1)
        mj0, n_e = meter.read(), 0
        while n_e < n_energy:
            step()
            n_e += 1
            if n_e % 4 == 0:
                torch.cuda.synchronize()
        torch.cuda.synchronize()
        mj1 = meter.read()
        joules = (mj1 - mj0) / 1e3 if mj0 is not None and mj1 is not None else float("nan")
        t = torch.tensor([joules, n_e], dtype=torch.float64, device=dev)
        if dist:
            dist.all_reduce(t, op=dist.ReduceOp.SUM)
            joules = float(t[0].item())
            n_e = int(t[1].item()) // ws
        if joules == joules and joules > 0 and n_e > 0:
            energy = {"joules_per_step": round(joules / n_e, 4),
                      "gpts_per_joule": round(points_job * sweeps * n_e / joules / 1e9, 3),
                      "steps": n_e, "note": "NVML total-energy counter, summed over GPUs, untimed steps"}

    # ---- per-pass breakdown and halo bandwidth (N > 1) ---------------------------------------
    pass_times = None
    halo = None
    if sharded:
        torch.cuda.synchronize()
        dist.barrier()
        _abi.check(lib.bst_comm_profile_begin(comm, 2 * sweeps))  # at most one pass per sweep
        for _ in range(2):
            step()
        out = (ctypes.c_double * 6)()
        _abi.check(lib.bst_comm_profile_end(comm, out))
        v = torch.tensor(list(out), dtype=torch.float64, device=dev)
        dist.all_reduce(v, op=dist.ReduceOp.MAX)
        npass = max(1.0, float(v[4].item()))
        slab_passes = max(1, int(round(npass / 2)))  # the library's own fusion, measured over two steps
        pass_times = {"boundary_ms": round(float(v[0].item()) / npass, 4),
                      "exchange_ms": round(float(v[1].item()) / npass, 4),
                      "interior_ms": round(float(v[2].item()) / npass, 4),
                      "span_ms": round(float(v[3].item()) / npass, 4),
                      "exposed_exchange_ms": round(float(v[5].item()) / npass, 4),
                      "passes": int(npass),
                      "note": "per pass, CUDA events on the boundary, comm and compute streams, two untimed steps, "
                              "max over ranks; exposed = exchange time left after the interior launch ended"}
        # NVLink halo bandwidth: one ghost exchange (G planes each way per neighbour) timed on
        # the device.  A sleep kernel ahead of it keeps the GPU busy while the host enqueues the
        # NCCL group, so the events bracket the exchange itself, not the host.
        times = []
        for _ in range(10):
            torch.cuda.synchronize()
            dist.barrier()
            h0, h1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            if hasattr(torch.cuda, "_sleep"):
                torch.cuda._sleep(2_000_000)
            h0.record(stream)
            _abi.check(lib.bst_halo_exchange(comm, ctypes.c_void_p(a.data_ptr()), dt, plane, n_local, G, sp))
            h1.record(stream)
            torch.cuda.synchronize()
            t = torch.tensor([h0.elapsed_time(h1)], dtype=torch.float64, device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            times.append(float(t.item()))
        ex_ms = statistics.median(times)
        nbrs = min(2, ws - 1)  # an interior rank's neighbours (an end rank's at N = 2)
        ex_bytes = 2 * nbrs * G * plane * es  # sent + received by that rank
        halo = {"transport": transport, "ghost_planes": G, "bytes_per_exchange": ex_bytes,
                "nccl_exchange_ms": round(ex_ms, 4), "nccl_nvlink_gbs": round(ex_bytes / (ex_ms * 1e-3) / 1e9, 2),
                "exchanges_per_step": slab_passes,
                "note": "nccl_*: one NCCL exchange of the ghost planes timed alone on the device after a sleep kernel "
                        "hides its host enqueue (median of 10, max over ranks)"}
        if transport == "copy":
            sent, cms = nbrs * G * plane * es, pass_times["exchange_ms"]
            halo.update({"copy_bytes_sent_per_pass": sent, "copy_ms": cms,
                         "copy_nvlink_gbs": round(sent / (cms * 1e-3) / 1e9, 2) if cms > 0 else None,
                         "copy_note": "per pass: cudaMemcpyAsync of the first and last ghost-depth owned planes "
                                      "into the neighbours' ghost planes (copy engines, peer mappings) plus the "
                                      "one-thread flag kernel, timed on the comm stream during the sweeps"})
        if transport == "peer":
            halo.update({"peer_bytes_stored_per_pass": nbrs * G * plane * es,
                         "peer_note": "one launch per sweep: the items holding the first and last ghost-depth "
                                      "owned planes copy them over NVLink into the neighbours' ghost planes at "
                                      "their end; the pass span is the whole cost, no separate exchange"})

    # Dominant kernel: the sweep; per pass over this rank's grid.
    passes = launches if not sharded else slab_passes * args.steps
    launch_ms = ms_total / max(1, passes)
    per_launch_bytes = 2 * es * local_points
    achieved = per_launch_bytes / (launch_ms * 1e-3) / 1e9
    peak, peak_src = _peaks()
    if w.name.startswith("mean3"):
        kernel = "line_kernel"
    elif sweeps * args.steps > passes:  # several sweeps fused per pass
        kernel = "march_tb3d_kernel" if len(gshape) == 3 else "march_tb2d_kernel"
    else:
        kernel = "march_tma_kernel"


    # ---- e2e through the public API with host buffers ---------------------------------------
    e2e = None
    if args.e2e_steps > 0 and not sharded:
        host_in = x0.cpu().pin_memory()
        out_shape = prog.out_shape(x0.shape)
        outs = [torch.empty(out_shape, dtype=w.dtype).pin_memory() for _ in range(E2E_SETS)]
        ex = [torch.empty_like(x0) for _ in range(E2E_SETS)]
        ea = [torch.empty(out_shape, dtype=w.dtype, device=dev) if prog.boundary == "zero" else None
              for _ in range(E2E_SETS)]
        eb = [torch.empty(out_shape, dtype=w.dtype, device=dev) for _ in range(E2E_SETS)]
        res = [None] * E2E_SETS

        def up(s):
            ex[s].copy_(host_in, non_blocking=True)

        def comp(s):
            res[s] = step_on(ex[s], ea[s], eb[s])

        def down(s):
            outs[s].copy_(res[s], non_blocking=True)

        e_ms = pipelined(args.e2e_steps, up, comp, down, stream)
        if dist:
            t = torch.tensor([e_ms], dtype=torch.float64, device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            e_ms = float(t.item())
        e2e = {"value": round(points_job * sweeps / (e_ms * 1e-3) / 1e9, 4), "unit": UNIT,
               "h2d_bytes_per_step": w.points * es * max(1, ws), "d2h_bytes_per_step": w.out_points * es * max(1, ws),
               "ms_per_step": round(e_ms, 3),
               "path": "basalto.apply + basalto.sweeps (C ABI bst_stencil_apply + bst_stencil_sweeps), pinned host "
                       "grid copied in and the result copied out every step; three buffer sets in flight, uploads and "
                       "downloads on separate copy streams" + ("; every rank a replica, max over ranks" if ws > 1 else "")}
        del ex, ea, eb
        torch.cuda.empty_cache()
        if ws == 1:
            # the drop-in plugin: torch.compile(backend="basalto") called once per sweep
            torch._dynamo.reset()
            cf = torch.compile(w.fn, backend="basalto")
            host_out = outs[0]

            def e2e_plugin():
                x = host_in.to(dev, non_blocking=True)
                y = x
                for _ in range(sweeps):
                    y = cf(y if prog.boundary == "zero" else x)
                host_out.copy_(y, non_blocking=True)

            e2e_plugin()
            torch.cuda.synchronize()
            f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            f0.record(stream)
            for _ in range(args.e2e_steps):
                e2e_plugin()
            f1.record(stream)
            torch.cuda.synchronize()
            p_ms = f0.elapsed_time(f1) / args.e2e_steps
            e2e["torch_compile_per_sweep"] = {"value": round(w.points * sweeps / (p_ms * 1e-3) / 1e9, 4),
                                              "ms_per_step": round(p_ms, 3)}
    elif args.e2e_steps > 0 and sharded:
        # The slab API with host buffers: each step copies this rank's owned planes in from
        # pinned host memory, exchanges their ghosts, runs the sweeps and copies the owned
        # result back.
        host_in = x0[G:G + n_local].cpu().pin_memory()
        outs = [torch.empty(local_shape, dtype=w.dtype).pin_memory() for _ in range(E2E_SETS)]
        sx = [x0] + [torch.zeros_like(x0) for _ in range(E2E_SETS - 1)]
        sa = [a] + [torch.zeros_like(a) for _ in range(E2E_SETS - 1)]
        sb = [b] + [torch.zeros_like(b) for _ in range(E2E_SETS - 1)]
        for k in range(1, E2E_SETS):
            register(sa[k])
            register(sb[k])
        res = [None] * E2E_SETS

        def up(s):
            sx[s][G:G + n_local].copy_(host_in, non_blocking=True)

        def comp(s):
            st = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
            _abi.check(lib.bst_halo_exchange(comm, ctypes.c_void_p(sx[s].data_ptr()), dt, plane, n_local, G, st))
            res[s] = step_on(sx[s], sa[s], sb[s])

        def down(s):
            outs[s].copy_(res[s][G:G + n_local], non_blocking=True)

        torch.cuda.synchronize()
        dist.barrier()
        t = torch.tensor([pipelined(args.e2e_steps, up, comp, down, stream)], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e_ms = float(t.item())
        total_bytes = int(np.prod(gshape)) * es
        e2e = {"value": round(points_job * sweeps / (e_ms * 1e-3) / 1e9, 4), "unit": UNIT,
               "h2d_bytes_per_step": total_bytes, "d2h_bytes_per_step": total_bytes,
               "ms_per_step": round(e_ms, 3),
               "path": "bst_halo_exchange + bst_slab_sweeps_deep per rank, pinned host slab copied in and out "
                       "each step (bytes summed over ranks), three buffer sets in flight, max over ranks"}

    # ---- CPU baseline (rank 0, N = 1 only, bounded sample) ------------------------------------
    cpu = None
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        ref = CpuReference(w, threads)
        r, secs, n = ref.rate_for(args.cpu_seconds)
        cpu = {"value": round(r, 4), "unit": UNIT, "cores": threads, "kind": "port",
               "sample": f"{n} sweeps ({secs:.1f} s): " + ref.describe()}

    if comm is not None:
        torch.cuda.synchronize()
        lib.bst_comm_destroy(comm)

    if rank == 0:
        scaling = "weak" if w.scaling in ("weak", "replicas") else "strong"
        line = {
            "metric": METRIC, "value": round(value, 4), "unit": UNIT, "n_gpus": ws, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_step, 4), "higher_is_better": True, "scaling": scaling,
            "vs_baseline": None, "dtype": _dtype_name(w), "data": "synthetic",
            "config": {"workload": w.label(),
                       "global_grid": "x".join(map(str, gshape)),
                       "parallelism": (f"z-slab x{ws} ({scaling} scaling, {G} ghost planes per side, "
                                       f"{TRANSPORT_NOTE[transport]})"
                                       if sharded
                                       else (f"{ws} independent replicas" if ws > 1 else "single GPU")),
                       "arithmetic": "fused multiply-add fold (BST_PROGRAM_CONTRACT)" if w.program.contract
                       else "separately rounded (bit-identical to eager torch)",
                       "l2": l2_note},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "peak_source": peak_src,
                         "frac_of_nominal_8000": round(achieved / 8000.0, 4),
                         "kernel": kernel, "traffic": _traffic(w.name, kernel),
                         "algorithmic_bytes_per_launch": per_launch_bytes, "avg_launch_ms": round(launch_ms, 5)},
            "parity": parity,
            "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": int(launches),
            "energy": energy, "passes": pass_times, "halo": halo,
            "sweeps_per_launch": round(sweeps * args.steps / max(1, passes), 3),
            "clocks": clk,
        }
        print(json.dumps(line), flush=True)
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    if not parity["ok"]:
        raise SystemExit(f"parity check failed: {bad} of {checked} sampled points differ from the oracle")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="basalto", choices=["basalto", "reference"])
    ap.add_argument("--workload", default=DEFAULT_WORKLOAD)
    ap.add_argument("--contract", action="store_true",
                    help="fold multiplied terms with fused multiply-add (BST_PROGRAM_CONTRACT) instead of "
                         "rounding every operation separately")
    ap.add_argument("--dtype", choices=["f32", "f64"], default=None,
                    help="override the workload's dtype (e.g. the 27-point box in fp32)")
    ap.add_argument("--shape", default="", help="override the workload's grid, e.g. 512x512x512")
    ap.add_argument("--cpu-seconds", type=float, default=10.0,
                    help="host work timed for the cpu_baseline field (whole sweeps, at least this long)")
    ap.add_argument("--e2e-steps", type=int, default=10,
                    help="end-to-end steps timed through the public API with host buffers (pipelined, three "
                         "buffer sets in flight); the first upload and last download are not overlapped, so "
                         "more steps approach the streaming rate")
    ap.add_argument("--transport", choices=["auto", "nccl", "copy", "peer"], default="auto",
                    help="N > 1 ghost planes: nccl = boundary planes first, NCCL exchange on a side stream while "
                         "the interior computes (deep halos where sweeps fuse); copy = the same passes with the "
                         "ghost planes pushed by the copy engines over NVLink; peer = one launch per sweep whose "
                         "boundary items store into the neighbours over NVLink; auto = nccl at 2 GPUs, copy "
                         "from 3 on")
    ap.add_argument("--ghost", type=int, default=0,
                    help="N > 1, NCCL or copy transport: ghost planes per side (a multiple of the axis-0 radius; default: "
                         "the library's fused depth).  Deeper ghosts let the slab sweeps fuse where a temporally "
                         "blocked kernel exists (3-D heat: 2 sweeps per exchange with 2 ghost planes)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    else:
        run_basalto(args)


if __name__ == "__main__":
    main()
