"""The "basalto" Dynamo backend without a GPU: registration, refusal of CPU tensors for
stencil graphs (no CPU fallback), and eager pass-through for non-stencil graphs — the
reference backend's behaviour for everything it does not run (compiler.py:44-75,95)."""
import pytest
import torch

import basalto  # noqa: F401  (registers the backend)
from basalto import workloads as W
from basalto.compiler import StencilCallable, basalto_backend


def test_backend_registered_under_reference_name():
    assert "basalto" in torch._dynamo.list_backends(exclude_tags=())


def test_stencil_graph_on_cpu_tensor_raises():
    torch._dynamo.reset()
    cf = torch.compile(W.heat7_3d, backend="basalto")
    with pytest.raises(Exception, match="CUDA"):
        cf(torch.rand(6, 7, 8))


def test_backend_returns_kernel_callable_for_stencils():
    graphs = []

    def spy(gm, ex):
        graphs.append(basalto_backend(gm, ex))
        return gm

    torch._dynamo.reset()
    torch.compile(W.jacobi5_2d, backend=spy)(torch.rand(8, 8))
    assert isinstance(graphs[0], StencilCallable)
    assert graphs[0].program_for([torch.rand(8, 8)])[0] == W.WORKLOADS["jacobi5_2d"].program


def test_non_stencil_graph_runs_eagerly(monkeypatch):
    monkeypatch.setenv("BASALTO_FALLBACK_EAGER", "1")
    torch._dynamo.reset()
    a, b = torch.randn(5, 6), torch.randn(6, 3)
    cf = torch.compile(lambda u, v: torch.matmul(u, v), backend="basalto")
    assert torch.equal(cf(a, b), a @ b)


def test_strict_mode_refuses_non_stencils(monkeypatch):
    monkeypatch.setenv("BASALTO_FALLBACK_EAGER", "0")
    torch._dynamo.reset()
    cf = torch.compile(lambda u: u * u, backend="basalto")
    with pytest.raises(Exception, match="not a supported stencil"):
        cf(torch.randn(4))
