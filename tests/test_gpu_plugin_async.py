"""The drop-in plugin path queues its work without waiting for the GPU.

`torch.compile(fn, backend="basalto")` hands every stencil call to the interceptor on torch's
current stream.  A program outside the compiled shape catalog runs the runtime-table kernel,
whose table is uploaded once per device and then reused, so a repeated call must neither copy
nor synchronise: here five calls are made while a ~2 s sleep kernel still occupies the stream,
and they must all return to the host long before it ends (any host synchronisation would wait
for it).  The results must still equal eager torch on the CPU bit for bit (eager CUDA torch
divides by a Python scalar as a multiplication by its reciprocal, so it is not the reference
for the division term).
"""
import time

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _odd_stencil(x):
    # Taps and terms no catalog shape has: a scaled diagonal pair, a divided corner tap, a bare sum.
    c = x[1:-1, 1:-1, 1:-1]
    d = x[2:, 2:, 1:-1] + x[:-2, 1:-1, :-2]
    return 0.3 * d + x[2:, :-2, 2:] / 7.0 + (c + x[1:-1, 2:, :-2])


def test_plugin_calls_return_before_the_gpu_finishes():
    import basalto  # noqa: F401  (registers the backend)
    if not hasattr(torch.cuda, "_sleep"):
        pytest.skip("this torch has no sleep kernel")
    torch._dynamo.reset()
    cf = torch.compile(_odd_stencil, backend="basalto")
    x = torch.rand(48, 40, 72, device="cuda", generator=torch.Generator(device="cuda").manual_seed(6))
    n0 = basalto.launch_count()
    y = cf(x)  # compiles, plans, uploads the program table
    torch.cuda.synchronize()
    assert basalto.launch_count() > n0, "the stencil did not run on the native kernels"
    torch.cuda._sleep(4_000_000_000)  # about two seconds of GPU time ahead of the calls
    t0 = time.perf_counter()
    for _ in range(5):
        y = cf(x)
    host_s = time.perf_counter() - t0
    torch.cuda.synchronize()
    assert host_s < 0.5, f"plugin calls waited for the GPU ({host_s:.2f} s on the host)"
    assert np.array_equal(y.cpu().numpy(), _odd_stencil(x.cpu()).numpy())
