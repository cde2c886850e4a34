"""Benchmark of the stencil hot path (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl basalto|reference] [--workload NAME]
    torchrun --nproc-per-node N bench.py --gpus N ...       (N > 1: one process per GPU)

Workload (default): 2-D five-point Jacobi, fp32 8192 x 8192 ~U(-1,1) seed 1, Dirichlet-0
ghost cells, 100 ping-pong sweeps.  One step = the full 100-sweep run.  At N > 1 every rank
owns an 8192 x 8192 slab of a (8192*N) x 8192 grid split along rows (weak scaling), with
deep ghosts: every fused pass of k sweeps exchanges k ghost rows with each neighbour over
NCCL, overlapped with the interior.

value      grid-point updates per second of the whole job (Gpts/s), inputs resident in HBM,
           CUDA events on the compute stream, max over ranks.  Inputs smaller than L2 are
           timed step by step with a 256 MiB write between steps.
e2e        the same metric through the public API with host buffers: every step copies the
           grid from pinned host memory, runs basalto.sweeps (C ABI bst_stencil_sweeps) and
           copies the result back, two steps in flight on separate copy streams.  At N > 1:
           bst_halo_exchange + bst_slab_sweeps_deep per rank with each slab copied in and out.
           e2e.torch_compile_per_sweep: torch.compile(fn, backend="basalto") called once per
           sweep (the drop-in plugin path).
roofline   the dominant kernel: algorithmic bytes (2 x element size per point: one read + one
           write) per pass over the grid / average pass time, against the measured HBM copy
           bandwidth; a temporally blocked pass performs several sweeps for those bytes.
halo       (N > 1) ghost planes, bytes and time of one exchange timed alone.
energy     NVML total-energy counter over the timed region, summed over ranks.
cpu_baseline / --impl reference
           the reference's CPU path: eager torch through the reference backend's control
           flow (oracle/reference_path.py), all host threads, ~10 s of sweeps.
--contract fused multiply-add arithmetic (BST_PROGRAM_CONTRACT); --dtype / --shape override
           the workload's element type / grid.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
for _p in (str(REPO), str(REPO / "bs-compiler_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import torch  # noqa: E402

METRIC = "stencil Gpts/s and % of HBM roofline at 1/2/4/8 B200 vs reference CPU path"
UNIT = "Gpts/s"
FALLBACK_HBM_GBS = 6650.0


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
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for name, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(name)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


class EnergyMeter:
    """NVML total-energy counter (millijoules since driver load) read around the timed region."""

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


def pipelined(n_steps, upload, compute, download, stream):
    """Time n_steps end-to-end steps with two buffer sets in flight.

    Step k uses set k % 2: its host->device upload runs on one copy stream, its compute on
    `stream`, its device->host download on a second copy stream (PCIe is full duplex), so step
    k+1's upload and step k-1's download overlap step k's compute.  Every step still copies its
    own input in and its own result out inside the timed region.  upload(s), compute(s) and
    download(s) enqueue on the current stream.  Returns ms per step (CUDA events on `stream`)."""
    h2d, d2h = torch.cuda.Stream(), torch.cuda.Stream()
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_done = [torch.cuda.Event() for _ in range(2)]
    ev_free = [None, None]

    def run(n):
        for k in range(n):
            s = k % 2
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

    run(2)  # warm-up
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
        dist.init_process_group(backend, rank=rank, world_size=ws, timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local) if backend == "nccl" else None)
    return dist


class CpuReference:
    """Eager torch on the host through the reference backend's control flow."""

    def __init__(self, workload, threads: int | None = None):
        from oracle.reference_path import compile_reference
        if threads:
            torch.set_num_threads(threads)
        self.w = workload
        self.x = workload.make_input()  # CPU, the configuration's own seeded grid
        self.cf = compile_reference(workload.fn)
        self.y = self.cf(self.x)  # compile + one warm sweep

    def rate_for(self, seconds: float, cap: int):
        """(Gpts/s, seconds, sweeps): consecutive sweeps until `seconds` of host work have run
        (at most `cap` sweeps).  Shrinking (valid-region) programs restart from the input."""
        chain = self.w.program.boundary == "zero"
        y = self.y if chain else self.x
        n = 0
        t0 = time.perf_counter()
        while True:
            out = self.cf(y)
            if chain:
                y = out
            n += 1
            dt = time.perf_counter() - t0
            if dt >= seconds or n >= cap:
                break
        if chain:
            self.y = y
        return self.w.points * n / dt / 1e9, dt, n

    def rate(self, sweeps: int):
        """(Gpts/s, seconds) over `sweeps` consecutive sweeps."""
        y = self.y
        t0 = time.perf_counter()
        for _ in range(sweeps):
            y = self.cf(y)
        dt = time.perf_counter() - t0
        self.y = y
        return self.w.points * sweeps / dt / 1e9, dt


def _workload(args):
    """The named workload, optionally on a different grid (--shape, e.g. for profiling)."""
    import dataclasses

    from basalto.workloads import WORKLOADS
    w = WORKLOADS[args.workload]
    if args.shape:
        w = dataclasses.replace(w, shape=tuple(int(v) for v in args.shape.split("x")))
    if args.dtype:
        w = dataclasses.replace(w, dtype={"f32": torch.float32, "f64": torch.float64}[args.dtype])
    if args.contract:  # fused multiply-add folding (the reference GPU kernel's arithmetic)
        w = dataclasses.replace(w, program=w.program.contracted())
        os.environ["BASALTO_FP_CONTRACT"] = "1"  # the torch.compile leg compiles the same program
    return w


def run_reference(args):
    ws, rank, local = _dist()
    from basalto.workloads import WORKLOADS
    w = _workload(args)
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    ref = CpuReference(w, threads)
    per_step = max(1, args.ref_sweeps)
    rates = []
    for i in range(args.warmup + args.steps):
        r, dt = ref.rate(per_step)
        if i >= args.warmup:
            rates.append((r, dt))
    value = statistics.median(r for r, _ in rates)
    ms = statistics.median(dt for _, dt in rates) * 1e3 / per_step * w.steps
    line = {
        "metric": METRIC, "value": round(value, 4), "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32" if w.dtype == torch.float32 else "f64",
        "data": "synthetic", "impl": "reference",
        "config": {"workload": f"{w.name} {'x'.join(map(str, w.shape))} {w.steps} sweeps",
                   "sample": f"{per_step} sweep(s) per step on the full grid; ms_per_step scaled to {w.steps} sweeps"},
        "cpu_baseline": {"value": round(value, 4), "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": f"{per_step} of {w.steps} sweeps per step, full {'x'.join(map(str, w.shape))} grid"},
        "e2e": {"value": round(value, 4), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_basalto(args):
    import ctypes

    import basalto
    from basalto import _abi
    from basalto.workloads import WORKLOADS

    ws, rank, local = _dist()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = _init_pg(ws, rank, local, "nccl") if ws > 1 else None
    w = _workload(args)
    prog = w.program
    sweeps = w.steps
    stream = torch.cuda.current_stream(dev)
    es = w.elem_size

    if ws == 1:
        a = w.make_input(device=dev)
        if prog.boundary == "zero":
            b = torch.empty_like(a)

            def step():
                basalto.sweeps(prog, a, b, sweeps)
        else:  # a shrinking (valid-region) stencil: one sweep per step into its own output
            b = torch.empty(prog.out_shape(a.shape), dtype=a.dtype, device=dev)

            def step():
                for _ in range(sweeps):
                    basalto.apply(prog, a, out=b)

        points_job = w.points
        comm = None
    else:
        # Weak scaling: each rank owns a full-size slab; deep ghost planes along axis 0 (the
        # fused kernel's k x radius, so one exchange per k sweeps).
        from basalto.slab import fuse_plan, slab_ghost_depth
        R = prog.radius()[0]
        local_shape = list(w.shape)
        dt = _abi.BST_F32 if w.dtype == torch.float32 else _abi.BST_F64
        G = slab_ghost_depth(prog, [local_shape[0] * ws] + local_shape[1:], ws, dt)
        g = torch.Generator(device=dev).manual_seed(w.seed + 1000 * rank)
        a = torch.zeros([local_shape[0] + 2 * G] + local_shape[1:], dtype=w.dtype, device=dev)
        b = torch.zeros_like(a)
        a[G:G + local_shape[0]].copy_(torch.rand(local_shape, generator=g, dtype=w.dtype, device=dev) * 2 - 1)
        uid = (ctypes.c_uint8 * 128)()
        obj = [None]
        if rank == 0:
            _abi.check(_abi.lib().bst_nccl_get_unique_id(uid))
            obj[0] = bytes(uid)
        dist.broadcast_object_list(obj, src=0)
        uid = (ctypes.c_uint8 * 128).from_buffer_copy(obj[0])
        h = ctypes.c_void_p()
        _abi.check(_abi.lib().bst_comm_create(uid, ws, rank, local, 120.0, ctypes.byref(h)))
        comm = h
        cp = prog.to_c(local_shape)
        plane = 1
        for s in local_shape[1:]:
            plane *= s
        sp = ctypes.c_void_p(stream.cuda_stream)
        _abi.check(_abi.lib().bst_halo_exchange(comm, ctypes.c_void_p(a.data_ptr()), dt, plane, local_shape[0], G, sp))
        shp = _abi.i64_array(local_shape)

        def step():
            _abi.check(_abi.lib().bst_slab_sweeps_deep(comm, ctypes.byref(cp), dt, len(local_shape), shp, G,
                                                       ctypes.c_void_p(a.data_ptr()), ctypes.c_void_p(b.data_ptr()),
                                                       sweeps, sp))

        # Passes over the slab per step (each pass = boundary launches + interior launch).
        slab_passes = len(fuse_plan(sweeps, G // R if R else 1))
        points_job = w.points * ws

    # ---- timed region (device time, CUDA events on the compute stream) -------------------
    l2_bytes = 126 << 20
    flush = None
    if w.points * es < l2_bytes:  # the input fits in L2: flush it between timed steps
        flush = torch.zeros(256 << 20, dtype=torch.uint8, device=dev)
        l2_note = "L2 flushed before every timed step (256 MiB write, outside the timed windows)"
    else:
        l2_note = f"inputs larger than L2 (2 x {w.points * es / 2**20:.0f} MiB ping-pong)"
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    clocks = ClockSampler(local)
    clocks.start()
    energy = EnergyMeter(local)
    mj0 = energy.read()
    n0 = basalto.launch_count()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    if flush is None:  # inputs larger than L2: consecutive steps cannot hit in L2
        e0.record(stream)
        for _ in range(args.steps):
            step()
        e1.record(stream)
        torch.cuda.synchronize()
        ms_total = e0.elapsed_time(e1)
    else:  # small inputs: L2 flushed before every step, each step timed on its own
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
        for a0, a1 in evs:
            flush.add_(1)  # writes 256 MiB (> L2) between timed steps
            a0.record(stream)
            step()
            a1.record(stream)
        torch.cuda.synchronize()
        ms_total = sum(a0.elapsed_time(a1) for a0, a1 in evs)
    if dist:
        dist.barrier()
    launches = basalto.launch_count() - n0
    mj1 = energy.read()
    clk = clocks.stop()
    joules = (mj1 - mj0) / 1e3 if mj0 is not None and mj1 is not None else float("nan")
    if dist:
        t = torch.tensor([joules], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        joules = float(t.item())
    if dist:
        t = torch.tensor([ms_total], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_total = float(t.item())
    ms_step = ms_total / args.steps
    value = points_job * sweeps * args.steps / (ms_total * 1e-3) / 1e9

    # Dominant kernel: the sweep itself; average launch = timed region / sweeps (per rank).
    # Multi-sweep runs fuse several sweeps per launch (temporal blocking); each launch still
    # reads its input grid once and writes its output once, so the algorithmic traffic of a
    # launch is 2 * elem bytes per point whatever the number of sweeps it fuses.
    # At N > 1 a pass over the slab is split into boundary and interior launches: the unit is
    # the pass (all of this rank's points once), timed over the whole region.
    passes = launches if ws == 1 else slab_passes * args.steps
    launch_ms = ms_total / max(1, passes)
    per_launch_bytes = 2 * es * w.points
    achieved = per_launch_bytes / (launch_ms * 1e-3) / 1e9
    peak, peak_src = _peaks()
    if w.name.startswith("mean3"):
        kernel = "line_kernel"
    elif sweeps * args.steps > passes:
        kernel = "march_tb2d_kernel"  # several sweeps fused per pass
    else:
        kernel = "march_tma_kernel"

    # ---- e2e through the public API with host buffers ---------------------------------------
    e2e = None
    if ws == 1 and args.e2e_steps > 0:
        host_in = w.make_input().pin_memory()
        host_out = torch.empty(prog.out_shape(w.shape), dtype=w.dtype).pin_memory()

        def timed(step_fn):
            step_fn()
            torch.cuda.synchronize()
            f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            f0.record(stream)
            for _ in range(args.e2e_steps):
                step_fn()
            f1.record(stream)
            torch.cuda.synchronize()
            return f0.elapsed_time(f1) / args.e2e_steps

        # (1) the multi-sweep call (basalto.sweeps -> bst_stencil_sweeps), host in and out, two
        #     steps in flight (uploads and downloads overlap the sweeps of the neighbouring steps)
        ea = [torch.empty(w.shape, dtype=w.dtype, device=dev) for _ in range(2)]
        eb = [torch.empty(prog.out_shape(w.shape), dtype=w.dtype, device=dev) for _ in range(2)]
        res = [None, None]
        outs = [host_out, torch.empty_like(host_out).pin_memory()]

        def up(s):
            ea[s].copy_(host_in, non_blocking=True)

        def comp(s):
            if prog.boundary == "zero":
                res[s] = basalto.sweeps(prog, ea[s], eb[s], sweeps)
            else:
                res[s] = basalto.apply(prog, ea[s], out=eb[s])

        def down(s):
            outs[s].copy_(res[s], non_blocking=True)

        e_ms = pipelined(args.e2e_steps, up, comp, down, stream)
        e2e = {"value": round(w.points * sweeps / (e_ms * 1e-3) / 1e9, 4), "unit": UNIT,
               "h2d_bytes_per_step": w.points * es, "d2h_bytes_per_step": w.out_points * es,
               "ms_per_step": round(e_ms, 3),
               "path": "basalto.sweeps (C ABI bst_stencil_sweeps), pinned host grid copied in and out each step; "
                       "two steps in flight on separate copy streams"}
        # (2) the drop-in plugin: torch.compile(backend="basalto") called once per sweep
        torch._dynamo.reset()
        cf = torch.compile(w.fn, backend="basalto")

        def e2e_plugin():
            x = host_in.to(dev, non_blocking=True)
            for _ in range(sweeps):
                x = cf(x)
            host_out.copy_(x, non_blocking=True)

        p_ms = timed(e2e_plugin)
        e2e["torch_compile_per_sweep"] = {"value": round(w.points * sweeps / (p_ms * 1e-3) / 1e9, 4),
                                          "ms_per_step": round(p_ms, 3)}

    halo = None
    if ws > 1:
        # NVLink halo bandwidth: one ghost exchange (G planes each way per neighbour) timed on
        # the device.  A ~1 ms sleep kernel ahead of it keeps the GPU busy while the host
        # enqueues the NCCL group, so the events bracket the exchange itself, not the host.
        n_ex = 10
        times = []
        for _ in range(n_ex):
            torch.cuda.synchronize()
            dist.barrier()
            h0, h1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            if hasattr(torch.cuda, "_sleep"):  # keeps the GPU busy while the host enqueues
                torch.cuda._sleep(2_000_000)
            h0.record(stream)
            _abi.check(_abi.lib().bst_halo_exchange(comm, ctypes.c_void_p(a.data_ptr()), dt, plane, local_shape[0],
                                                    G, sp))
            h1.record(stream)
            torch.cuda.synchronize()
            t = torch.tensor([h0.elapsed_time(h1)], dtype=torch.float64, device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            times.append(float(t.item()))
        ex_ms = statistics.median(times)
        nbrs = min(2, ws - 1)  # an interior rank's neighbours (an end rank's at N = 2)
        ex_bytes = 2 * nbrs * G * plane * es  # sent + received by that rank
        halo = {"ghost_planes": G, "bytes_per_exchange": ex_bytes, "exchange_ms": round(ex_ms, 4),
                "nvlink_gbs": round(ex_bytes / (ex_ms * 1e-3) / 1e9, 2),
                "exchanges_per_step": slab_passes,
                "note": "one exchange timed on the device after a sleep kernel hides its host enqueue "
                        "(median of 10, max over ranks); in the sweep loop it overlaps the interior launch"}

    if ws > 1 and args.e2e_steps > 0:
        # The slab API with host buffers: each step copies this rank's slab in from pinned host
        # memory, exchanges ghosts, runs the sweeps and copies the owned result back.
        host_in = (torch.rand(local_shape, generator=torch.Generator().manual_seed(w.seed + rank), dtype=w.dtype)
                   * 2 - 1).pin_memory()
        outs = [torch.empty(local_shape, dtype=w.dtype).pin_memory() for _ in range(2)]
        sa = [a, torch.zeros_like(a)]
        sb = [b, torch.zeros_like(b)]
        nl = local_shape[0]

        def up(s):
            sa[s][G:G + nl].copy_(host_in, non_blocking=True)

        def comp(s):
            _abi.check(_abi.lib().bst_halo_exchange(comm, ctypes.c_void_p(sa[s].data_ptr()), dt, plane, nl, G, sp))
            _abi.check(_abi.lib().bst_slab_sweeps_deep(comm, ctypes.byref(cp), dt, len(local_shape), shp, G,
                                                       ctypes.c_void_p(sa[s].data_ptr()),
                                                       ctypes.c_void_p(sb[s].data_ptr()), sweeps, sp))

        def down(s):
            res = sa[s] if sweeps % 2 == 0 else sb[s]
            outs[s].copy_(res[G:G + nl], non_blocking=True)

        torch.cuda.synchronize()
        dist.barrier()
        t = torch.tensor([pipelined(args.e2e_steps, up, comp, down, stream)], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e_ms = float(t.item())
        e2e = {"value": round(points_job * sweeps / (e_ms * 1e-3) / 1e9, 4), "unit": UNIT,
               "h2d_bytes_per_step": w.points * es * ws, "d2h_bytes_per_step": w.points * es * ws,
               "ms_per_step": round(e_ms, 3),
               "path": "bst_halo_exchange + bst_slab_sweeps_deep per rank, pinned host slab copied in and out "
                       "each step (bytes summed over ranks), two steps in flight, max over ranks"}

    # ---- CPU baseline (rank 0, N = 1 only, bounded sample) ------------------------------------
    cpu = None
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        r, dt, n = CpuReference(w, threads).rate_for(args.cpu_seconds, cap=100000)
        cpu = {"value": round(r, 4), "unit": UNIT, "cores": threads, "kind": "port",
               "sample": f"{n} consecutive sweeps ({dt:.1f} s) on the full {'x'.join(map(str, w.shape))} grid "
                         f"({sweeps} sweeps per step), eager torch via the reference backend's control flow"}

    if comm is not None:
        torch.cuda.synchronize()
        _abi.lib().bst_comm_destroy(comm)

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 4), "unit": UNIT, "n_gpus": ws, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_step, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32" if w.dtype == torch.float32 else "f64", "data": "synthetic",
            "config": {"workload": f"{w.name} {'x'.join(map(str, w.shape))}{' per GPU' if ws > 1 else ''}, "
                                   f"{sweeps} sweeps per step",
                       "parallelism": f"z-slab x{ws}" if ws > 1 else "single GPU",
                       "arithmetic": "fused multiply-add fold (BST_PROGRAM_CONTRACT)" if w.program.contract
                       else "separately rounded (bit-identical to eager torch)",
                       "l2": l2_note},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "peak_source": peak_src,
                         "frac_of_nominal_8000": round(achieved / 8000.0, 4),
                         "kernel": kernel, "traffic": _traffic(w.name, kernel),
                         "algorithmic_bytes_per_launch": per_launch_bytes, "avg_launch_ms": round(launch_ms, 5)},
            "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": int(launches),
            "energy": {"joules_per_step": round(joules / args.steps, 4),
                       "gpts_per_joule": round(points_job * sweeps * args.steps / joules / 1e9, 3)}
                      if joules == joules and joules > 0 else None,
            "halo": halo,
            "sweeps_per_launch": round(sweeps * args.steps / max(1, launches), 3),
            "clocks": clk,
        }
        print(json.dumps(line), flush=True)
    if dist:
        dist.barrier()
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="basalto", choices=["basalto", "reference"])
    ap.add_argument("--workload", default="jacobi5_2d")
    ap.add_argument("--contract", action="store_true",
                    help="fold multiplied terms with fused multiply-add (BST_PROGRAM_CONTRACT) instead of "
                         "rounding every operation separately")
    ap.add_argument("--dtype", choices=["f32", "f64"], default=None,
                    help="override the workload's dtype (e.g. the 27-point box in fp32)")
    ap.add_argument("--shape", default="", help="override the workload's grid, e.g. 512x512x512")
    ap.add_argument("--ref-sweeps", type=int, default=3, help="sweeps per step of --impl reference")
    ap.add_argument("--cpu-seconds", type=float, default=10.0,
                    help="host work timed for the cpu_baseline field (whole sweeps, at least this long)")
    ap.add_argument("--e2e-steps", type=int, default=3)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--host-input", action="store_true", default=True)
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    else:
        run_basalto(args)


if __name__ == "__main__":
    main()
