"""Generate the golden fixtures in this directory from the reference's own backend.

    python tests/golden/make_golden.py --reference PATH_TO_REFERENCE_CHECKOUT

Runs in the development container, where the reference source tree is mounted; the GPU box
and the tests only read the committed .npz files.

For every case the stencil function is compiled with the reference's Dynamo backend
(`basalto_backend` from python/basalto/compiler.py of the reference) on seeded CPU inputs.
Its Rust interceptor cannot be built (no Rust toolchain, and the workspace does not build),
so `basalto._rust` is replaced by a recorder: the reference only uses that call to fill a
discarded buffer (compiler.py:78-95), and the recorder keeps the arguments it would have
received.  The value the reference returns to the user is the graph run eagerly — that is
the golden output.  The module-level `torch._dynamo.register_backend("basalto",
basalto_backend)` of the reference (compiler.py:97) passes its arguments in the wrong order
and raises on import under torch 2.x; the backend function itself is already defined by
then and is used directly.

Cases: the five workload functions of this package at small sizes (several shapes, single
sweeps and multi-sweep runs), and the stencil functions of the reference's own report
scripts (report/scripts/stencil_benchmark.py:make_stencil_fn, energy_benchmark.py:stencil_3d
and the stencil of multi_gpu_halo.py), together with the program this package's FX
extractor derives from each Dynamo graph.
"""
from __future__ import annotations

import argparse
import ast
import importlib.util
import json
import sys
import textwrap
import types
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
PKG_DIR = REPO / "bs-compiler_b200" / "basalto"


def _load_package_modules():
    """Import this package's pure-Python modules without its native extension."""
    name = "b200_golden_pkg"
    spec = importlib.util.spec_from_file_location(name, PKG_DIR / "__init__.py",
                                                  submodule_search_locations=[str(PKG_DIR)])
    pkg = importlib.util.module_from_spec(spec)
    sys.modules[name] = pkg  # __init__ is not executed: no native library is loaded
    out = {}
    for sub in ("_abi", "program", "workloads", "fx_extract"):
        s = importlib.util.spec_from_file_location(f"{name}.{sub}", PKG_DIR / f"{sub}.py")
        m = importlib.util.module_from_spec(s)
        sys.modules[f"{name}.{sub}"] = m
        s.loader.exec_module(m)
        out[sub] = m
    return out


class _Recorder:
    calls: list = []

    def compile_and_execute(self, **kw):
        _Recorder.calls.append({k: v for k, v in kw.items() if not k.startswith("device_ptr_") or k == "device_ptr_z"})


def _load_reference_backend(ref: Path):
    saved = {k: sys.modules.get(k) for k in ("basalto", "basalto._rust", "basalto.compiler")}
    pkg = types.ModuleType("basalto")
    pkg.__path__ = []
    rust = types.ModuleType("basalto._rust")
    rust.PyBasaltoInterceptor = _Recorder
    pkg._rust = rust
    sys.modules["basalto"] = pkg
    sys.modules["basalto._rust"] = rust
    spec = importlib.util.spec_from_file_location("basalto.compiler", ref / "python" / "basalto" / "compiler.py")
    m = importlib.util.module_from_spec(spec)
    try:
        spec.loader.exec_module(m)
        note = "imported cleanly"
    except AssertionError:
        note = "module-level register_backend raised AssertionError (argument order); backend function used directly"
    for k, v in saved.items():
        if v is None:
            sys.modules.pop(k, None)
        else:
            sys.modules[k] = v
    return m.basalto_backend, note


def _load_reference_report_fns(ref: Path):
    sys.path.insert(0, str(ref / "report"))
    try:
        sb = importlib.util.spec_from_file_location("ref_stencil_benchmark", ref / "report" / "scripts" / "stencil_benchmark.py")
        stencil_benchmark = importlib.util.module_from_spec(sb)
        sb.loader.exec_module(stencil_benchmark)
        eb = importlib.util.spec_from_file_location("ref_energy_benchmark", ref / "report" / "scripts" / "energy_benchmark.py")
        energy_benchmark = importlib.util.module_from_spec(eb)
        eb.loader.exec_module(energy_benchmark)
    finally:
        sys.path.pop(0)
    # The multi-GPU script defines its stencil inside a function; take it from the source.
    src = (ref / "report" / "scripts" / "multi_gpu_halo.py").read_text()
    tree = ast.parse(src)
    fn_src = None
    for node in ast.walk(tree):
        if isinstance(node, ast.FunctionDef) and node.name == "stencil_fn":
            fn_src = textwrap.dedent(ast.get_source_segment(src, node))
    ns = {}
    exec(compile(fn_src, "multi_gpu_halo.py:stencil_fn", "exec"), ns)  # noqa: S102
    return stencil_benchmark.make_stencil_fn, stencil_benchmark.make_stencil_coeffs, energy_benchmark.stencil_3d, ns["stencil_fn"]


def _program_json(prog):
    return json.dumps({
        "ndim": prog.ndim, "init_zero": prog.init_zero, "boundary": prog.boundary, "shrink": list(prog.shrink),
        "terms": [[t.op, t.scale, [list(o) for o in t.taps]] for t in prog.terms],
    })


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="root of a basaltotech/bs-compiler checkout")
    args = ap.parse_args()
    ref = Path(args.reference)
    torch.set_num_threads(1)
    mods = _load_package_modules()
    W = mods["workloads"]
    FX = mods["fx_extract"]
    backend, note = _load_reference_backend(ref)
    make_stencil_fn, make_stencil_coeffs, energy_stencil_3d, halo_stencil_fn = _load_reference_report_fns(ref)

    captured = []

    def run(fn, x, steps=1):
        """Compile with the reference backend; return (output after `steps` calls, FX program)."""
        torch._dynamo.reset()
        graphs = []

        def spy(gm, ex):
            graphs.append((gm, list(ex)))
            return backend(gm, ex)

        cf = torch.compile(fn, backend=spy)
        y = x
        for _ in range(steps):
            y = cf(y)
        prog = None
        gm, ex = graphs[0]
        try:
            prog, _ = FX.extract(gm, ex)
        except FX.Unsupported as e:
            print("  extractor:", e)
        return y, prog

    cases = []
    wl = W.WORKLOADS

    def add_case(name, fn, x, steps=1, extra=None):
        _Recorder.calls.clear()
        y, prog = run(fn, x, steps)
        rec = _Recorder.calls[0] if _Recorder.calls else {}
        rec = {k: (list(v) if isinstance(v, (tuple, list)) else v) for k, v in rec.items()}
        cases.append((name, x, y, prog, rec, steps, extra or {}))
        print(f"{name}: in {tuple(x.shape)} {x.dtype} steps={steps} -> out {tuple(y.shape)}; "
              f"program {'yes' if prog else 'no'}; reference call {rec.get('op')} {rec.get('dtype')}")

    g = W.gen_input
    # Workloads at small sizes (same distributions and seeds as the full configurations).
    for shape in [(1000,), (1,), (3,), (37,)]:
        add_case(f"mean3_1d_{'x'.join(map(str, shape))}", wl["mean3_1d"].fn, g("randn", shape, torch.float32, 0))
    for shape, steps in [((37, 45), 1), ((64, 64), 1), ((3, 200), 1), ((1, 1), 1), ((40, 33), 5)]:
        add_case(f"jacobi5_2d_{shape[0]}x{shape[1]}_s{steps}", wl["jacobi5_2d"].fn,
                 g("rand_pm1", shape, torch.float32, 1), steps)
    for shape, steps in [((19, 23, 29), 1), ((8, 16, 32), 1), ((2, 3, 5), 1), ((12, 17, 40), 3)]:
        add_case(f"heat7_3d_{'x'.join(map(str, shape))}_s{steps}", wl["heat7_3d"].fn,
                 g("rand", shape, torch.float32, 2), steps)
    w27 = W.box27_weights(3)
    for shape, steps in [((13, 17, 19), 1), ((6, 9, 16), 2)]:
        add_case(f"box27_3d_{'x'.join(map(str, shape))}_s{steps}", W.make_box27_3d(w27),
                 g("randn", shape, torch.float64, 3), steps, {"weights": w27})
    for shape, steps in [((12, 14, 33), 1), ((6, 5, 9), 1), ((16, 16, 16), 2)]:
        add_case(f"star25_3d_{'x'.join(map(str, shape))}_s{steps}", W.make_star_3d(),
                 g("randn", shape, torch.float32, 4), steps)
    # The reference's own report stencils.
    for dims, shape in [(1, (100,)), (2, (20, 30)), (3, (9, 10, 11))]:
        coeffs = make_stencil_coeffs(dims, 1, 2)
        add_case(f"ref_roll_box_{dims}d_r1", make_stencil_fn(dims, 1, coeffs), g("randn", shape, torch.float32, 5))
    add_case("ref_roll_box_2d_r2", make_stencil_fn(2, 2, make_stencil_coeffs(2, 2, 4)),
             g("randn", (21, 26), torch.float32, 6))
    add_case("ref_energy_stencil_3d", energy_stencil_3d, g("randn", (12, 13, 14), torch.float32, 7))
    add_case("ref_multi_gpu_halo_stencil", halo_stencil_fn, g("randn", (12, 13, 14), torch.float32, 8))

    arrays = {}
    meta = {"generator": "tests/golden/make_golden.py", "reference_backend": note, "torch": torch.__version__,
            "cases": []}
    for name, x, y, prog, rec, steps, extra in cases:
        arrays[f"{name}__in"] = x.numpy()
        arrays[f"{name}__out"] = y.detach().numpy()
        meta["cases"].append({"name": name, "steps": steps, "program": json.loads(_program_json(prog)) if prog else None,
                              "reference_call": rec, **extra})
    out = HERE / "stencils.npz"
    np.savez_compressed(out, meta=np.array(json.dumps(meta)), **arrays)
    print("wrote", out, out.stat().st_size, "bytes")


if __name__ == "__main__":
    main()
