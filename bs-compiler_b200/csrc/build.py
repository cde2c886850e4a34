"""In-tree build of the native parts of the package.

    python bs-compiler_b200/csrc/build.py [-v] [--force]

Produces, next to the Python package (so they ship with the source tree):
  bs-compiler_b200/basalto/libbasalto_b200.so   C ABI (include/basalto_b200.h) + sm_100a kernels
  bs-compiler_b200/basalto/_rust<EXT_SUFFIX>    the `basalto._rust` extension module
Kernels are compiled for sm_100a only.  FP contraction is disabled (-fmad=false) and the
kernels use explicitly rounded intrinsics, so no multiply-add is ever fused.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import subprocess
import sys
import sysconfig
from pathlib import Path

CSRC = Path(__file__).resolve().parent
PKG_ROOT = CSRC.parent
PKG = PKG_ROOT / "basalto"
REPO = PKG_ROOT.parent
INCLUDE = REPO / "include"
OBJ = PKG_ROOT / "_build"

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
CUDA_HOME = Path(NVCC).resolve().parent.parent
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVFLAGS = ARCH + ["-O3", "-std=c++17", "-lineinfo", "-fmad=false", "--expt-relaxed-constexpr",
                  "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden", f"-I{INCLUDE}"]
NVFLAGS += os.environ.get("BST_NVCC_EXTRA", "").split()  # e.g. tile-size macros for tuning builds

KERNEL_UNITS = ["bst_core.cu", "bst_f32.cu", "bst_f64.cu", "bst_interceptor.cu", "bst_halo.cu", "bst_noalloc.cu"]
HEADERS = sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + [INCLUDE / "basalto_b200.h"]

LIB = PKG / "libbasalto_b200.so"
EXT = PKG / ("_rust" + sysconfig.get_config_var("EXT_SUFFIX"))


def _newer(out: Path, deps) -> bool:
    if not out.exists():
        return False
    t = out.stat().st_mtime
    return all(Path(d).stat().st_mtime <= t for d in deps)


def _run(cmd, verbose):
    if verbose:
        print(" ".join(str(c) for c in cmd), flush=True)
    r = subprocess.run([str(c) for c in cmd], capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"build step failed ({r.returncode}): {' '.join(map(str, cmd))}\n{r.stdout}\n{r.stderr}")
    return r


def build(verbose: bool = False, force: bool = False) -> list[Path]:
    OBJ.mkdir(parents=True, exist_ok=True)
    objs = []
    jobs = []
    for unit in KERNEL_UNITS:
        src = CSRC / unit
        obj = OBJ / (unit + ".o")
        objs.append(obj)
        if force or not _newer(obj, [src, *HEADERS]):
            jobs.append([NVCC, *NVFLAGS, "-c", src, "-o", obj])
    if jobs:
        with cf.ThreadPoolExecutor(max_workers=min(len(jobs), os.cpu_count() or 4)) as ex:
            for f in [ex.submit(_run, j, verbose) for j in jobs]:
                f.result()
    if force or jobs or not _newer(LIB, objs):
        # Visibility: the C ABI is exported via extern "C" + default visibility below.
        _run([NVCC, *ARCH, "-shared", "-o", LIB, *objs, "-Xcompiler", "-fPIC", "-lcudart_static", "-ldl",
              "-lpthread", "-lrt", "-Xlinker", "--version-script=" + str(CSRC / "exports.map")], verbose)
    import pybind11  # noqa: WPS433  (build-time dependency)

    py_inc = sysconfig.get_paths()["include"]
    if force or not _newer(EXT, [CSRC / "py_rust.cpp", LIB, INCLUDE / "basalto_b200.h"]):
        _run(["g++", "-O2", "-std=c++17", "-shared", "-fPIC", "-fvisibility=hidden", f"-I{pybind11.get_include()}",
              f"-I{py_inc}", f"-I{INCLUDE}", CSRC / "py_rust.cpp", "-o", EXT, f"-L{PKG}", "-lbasalto_b200",
              "-Wl,-rpath,$ORIGIN"], verbose)
    return [LIB, EXT]


if __name__ == "__main__":
    out = build(verbose="-v" in sys.argv, force="--force" in sys.argv)
    for p in out:
        print(p)
