"""Test configuration: import paths, the `gpu` marker and shared fixtures."""
from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parent.parent
for p in (REPO, REPO / "bs-compiler_b200"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))

GOLDEN = REPO / "tests" / "golden" / "stencils.npz"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); run with -m gpu")


def pytest_collection_modifyitems(config, items):
    try:
        import torch
        has_cuda = torch.cuda.is_available()
    except Exception:  # pragma: no cover
        has_cuda = False
    if has_cuda:
        return
    skip = pytest.mark.skip(reason="no CUDA device visible")
    for it in items:
        if "gpu" in it.keywords:
            it.add_marker(skip)


class Golden:
    def __init__(self, path=GOLDEN):
        self._z = np.load(path)
        self.meta = json.loads(str(self._z["meta"]))
        self.cases = {c["name"]: c for c in self.meta["cases"]}

    def input(self, name):
        return self._z[f"{name}__in"]

    def output(self, name):
        return self._z[f"{name}__out"]

    def terms(self, name):
        p = self.cases[name]["program"]
        return [(op, s, [tuple(o) for o in taps]) for op, s, taps in p["terms"]]


@pytest.fixture(autouse=True)
def _device_errors_clean(request):
    """After every GPU test: no kernel may have given up a bounded wait."""
    yield
    if "gpu" in request.keywords:
        import torch
        if torch.cuda.is_available():
            import basalto
            basalto.check_device_errors()


@pytest.fixture(scope="session")
def golden():
    return Golden()


def program_from_meta(p):
    """StencilProgram from a fixture's program record."""
    from basalto.program import StencilProgram, Term
    return StencilProgram(p["ndim"], tuple(Term(op, s, tuple(tuple(o) for o in taps)) for op, s, taps in p["terms"]),
                          init_zero=p["init_zero"], boundary=p["boundary"], shrink=tuple(p["shrink"]))


def oracle_terms(prog):
    return [(t.op, t.scale, t.taps) for t in prog.terms]
