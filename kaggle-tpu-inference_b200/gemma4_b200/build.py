"""Build the sm_100a C-ABI library ``libg4b200.so`` in-tree with nvcc.

The library is compiled directly for ``sm_100a`` (B200); nvcc cross-compiles on a
machine without a GPU.  ``python -m gemma4_b200.build`` (from the package's parent
directory) or :func:`build` rebuilds only when a source is newer than the library.
"""

from __future__ import annotations

import glob
import os
import shutil
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG_DIR)                      # kaggle-tpu-inference_b200/
CSRC = os.path.join(ROOT, "csrc")
INCLUDE = os.path.join(os.path.dirname(ROOT), "include")
LIB = os.path.join(PKG_DIR, "libg4b200.so")
LIB_TRACE = os.path.join(PKG_DIR, "libg4b200_trace.so")  # -DG4_TRACE timeline build

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-shared",
]


def sources() -> list[str]:
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cuh"))
                  + glob.glob(os.path.join(INCLUDE, "*.h")))


def nvcc() -> str:
    path = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(path):
        raise RuntimeError("nvcc not found: the g4b200 library cannot be built")
    return path


def up_to_date(lib: str = LIB) -> bool:
    if not os.path.exists(lib):
        return False
    t = os.path.getmtime(lib)
    return all(os.path.getmtime(s) <= t for s in sources())


def _headers() -> list[str]:
    return sorted(glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(INCLUDE, "*.h")))


def build(force: bool = False, verbose: bool = False, trace: bool = False, jobs: int = 0) -> str:
    """Compile the library (``trace=True``: the -DG4_TRACE timeline build).

    Every translation unit (the runtime, and one per persistent step-kernel variant)
    is compiled to its own object in parallel, then linked; objects newer than their
    source and every header are reused.
    """
    lib = LIB_TRACE if trace else LIB
    if not force and up_to_date(lib):
        return lib
    objdir = os.path.join(PKG_DIR, "_build_trace" if trace else "_build")
    os.makedirs(objdir, exist_ok=True)
    units = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    newest_header = max(os.path.getmtime(h) for h in _headers())
    extra = ["-DG4_TRACE"] if trace else []
    compile_flags = [f for f in NVCC_FLAGS if f != "-shared"]

    def obj_of(u: str) -> str:
        return os.path.join(objdir, os.path.basename(u)[:-3] + ".o")

    def compile_one(u: str) -> None:
        o = obj_of(u)
        if not force and os.path.exists(o) and os.path.getmtime(o) >= max(os.path.getmtime(u), newest_header):
            return
        cmd = [nvcc(), *compile_flags, *extra, "-I", INCLUDE, "-c", "-o", o + ".tmp", u]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
        os.replace(o + ".tmp", o)

    from concurrent.futures import ThreadPoolExecutor

    with ThreadPoolExecutor(max_workers=jobs or os.cpu_count() or 4) as ex:
        list(ex.map(compile_one, units))
    tmp = lib + ".tmp"
    cmd = [nvcc(), "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-o", tmp,
           *[obj_of(u) for u in units]]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    os.replace(tmp, lib)
    return lib


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True, trace="--trace" in sys.argv))
