"""basalto — B200-native stencil hot path of the Basalto JIT compiler.

`import basalto` registers the `"basalto"` torch.compile backend (as the reference's
package does, python/basalto/compiler.py:97) and exposes:

  basalto._rust.PyBasaltoInterceptor   the reference's operator boundary (C++ host)
  basalto.apply(prog, x, out=None)     one sweep of a StencilProgram on a CUDA tensor
  basalto.sweeps(prog, a, b, n)        n ping-pong sweeps without host round trips
  basalto.program / basalto.workloads  stencil programs and the measured workloads

The native library is required: importing fails if it has not been built
(bs-compiler_b200/csrc/build.py); there is no CPU fallback.
"""
from __future__ import annotations

from . import _rust  # noqa: F401  (fails loudly when the extension is missing)
from . import _abi
from .api import apply, sweeps, launch_count, device_caps, cache_key, check_device_errors  # noqa: F401
from .compiler import basalto_backend  # noqa: F401  (registers the backend)
from .program import StencilProgram, Term  # noqa: F401

__all__ = ["apply", "sweeps", "launch_count", "check_device_errors", "device_caps", "cache_key", "basalto_backend",
           "StencilProgram", "Term"]
