"""Host-side pieces of bench.py: the sampled parity check and the reference arm's isolation.

The bench checks its result at sampled points by folding each point's input neighbourhood
with the oracle (bench.oracle_at_point); here that shortcut is compared with the oracle run
on the whole grid.  The reference arm must time the reference's CPU path without mapping any
native library of this repository.
"""
import json
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

import bench
from oracle import stencil_oracle as O

REPO = Path(__file__).resolve().parent.parent


def _programs():
    from basalto import program as P
    return {
        "star25": P.star_3d(P.LAPLACIAN8_COEFFS),
        "heat7": P.heat7_3d(),
        "box27": P.box(3, 1, [float(v) for v in np.linspace(0.01, 0.03, 27)]),
        "jacobi": P.jacobi5_2d(),
    }


@pytest.mark.parametrize("name,shape,sweeps", [("star25", (22, 19, 23), 2), ("heat7", (12, 13, 14), 4),
                                               ("box27", (9, 10, 11), 3), ("jacobi", (30, 27), 6)])
def test_neighbourhood_oracle_equals_whole_grid(name, shape, sweeps):
    prog = _programs()[name]
    terms = [(t.op, t.scale, t.taps) for t in prog.terms]
    x = np.random.default_rng(3).standard_normal(shape).astype(np.float32)
    full = x
    for _ in range(sweeps):
        full = O.eval_program(full, terms, prog.init_zero, "zero")
    xt = torch.from_numpy(x)
    reach = [r * sweeps for r in prog.radius()]
    owners = [bench_part for bench_part in [(0, shape[0] // 2), (shape[0] // 2, shape[0] - shape[0] // 2)]]
    pts = bench.sample_points(shape, owners, seed=5, n_random=6)
    # corners, rank boundaries and interior points all appear
    zs = {p[0] for p in pts}
    assert {0, shape[0] - 1, shape[0] // 2 - 1, shape[0] // 2} <= zs
    for p in pts:
        box, lo = bench.neighbourhood(xt, p, reach)
        got = bench.oracle_at_point(box, lo, shape, p, prog, sweeps)
        assert np.array_equal(np.asarray(got), full[p]), p


def test_reference_arm_maps_no_native_library():
    """The reference arm's workload table loads program.py/workloads.py without the package
    __init__, so none of this repository's .so files is mapped."""
    code = ("import sys, json; sys.path.insert(0, %r); import bench; t = bench._workload_table(False); "
            "w = t['star25_3d']; print(json.dumps({'maps': bench._native_maps(), 'label': w.label()}))" % str(REPO))
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    d = json.loads(r.stdout.strip().splitlines()[-1])
    assert d["maps"] == []
    from basalto.workloads import WORKLOADS
    assert d["label"] == WORKLOADS["star25_3d"].label()  # both arms name the configuration alike


def test_cpu_sample_is_bounded():
    from basalto.workloads import WORKLOADS
    assert bench.cpu_sample_shape(WORKLOADS["star25_3d"]) == (64, 1024, 1024)
    assert bench.cpu_sample_shape(WORKLOADS["jacobi5_2d"]) == (2048, 8192)
    assert bench.cpu_sample_shape(WORKLOADS["mean3_1d"]) == (1 << 24,)
    assert WORKLOADS["box27_3d"].global_shape(8) == (6144, 768, 768)
    assert WORKLOADS["star25_3d"].global_shape(8) == (1024, 1024, 1024)
