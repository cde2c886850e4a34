"""The reference's CPU path, restated for timing — TEST/BASELINE INFRASTRUCTURE ONLY.

The reference's Dynamo backend (python/basalto/compiler.py:6-95) classifies the graph by
substring-matching FX targets (compiler.py:10-40), allocates a throw-away
`y = torch.zeros_like(x)` (compiler.py:78), hands raw pointers to its Rust interceptor and
returns the unmodified graph (compiler.py:95), so each call of the compiled function runs
the user's stencil as eager PyTorch ops.  `reference_backend` reproduces that control flow;
the interceptor call is omitted because its output buffer is discarded (and its Rust side
cannot be built here).  Used by bench.py's `--impl reference` arm and its `cpu_baseline`
leg, on CPU tensors with all host threads.
"""
from __future__ import annotations

import torch


def _classify(gm) -> str:
    """compiler.py:10-40: the first call_function target containing matmul/mm/bmm,
    attention or softmax decides; everything else is "stencil"."""
    for node in gm.graph.nodes:
        if node.op == "call_function":
            t = str(node.target)
            if "matmul" in t or "mm" in t or "bmm" in t:
                return "matmul"
            if "attention" in t:
                return "attention"
            if "softmax" in t:
                return "softmax"
    return "stencil"


def reference_backend(gm, example_inputs):
    if not example_inputs:
        return gm
    if _classify(gm) == "stencil":
        x = example_inputs[0]
        _ = torch.zeros_like(x)  # the discarded output buffer of compiler.py:78
    return gm


def compile_reference(fn):
    """fn compiled through the reference backend for one static shape (dynamic=False), so a
    process that already compiled fn for another grid does not hand the backend symbolic
    sizes."""
    torch._dynamo.reset()
    return torch.compile(fn, backend=reference_backend, dynamic=False)
