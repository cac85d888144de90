"""Build ``libphmoe.so`` (the C-ABI library) in-tree with nvcc for sm_100a.

Usage: ``python -m phantom_moe._build`` (from ``solution-is-all-you-need_b200``)
or ``phantom_moe._build.build()``. Objects go to ``_build/`` next to the
package; the library to ``phantom_moe/lib/libphmoe.so``. Sources are only
recompiled when they (or a header) changed.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
SRC_ROOT = PKG_DIR.parent                      # solution-is-all-you-need_b200/
CSRC = SRC_ROOT / "csrc"
REPO = SRC_ROOT.parent
INCLUDE = REPO / "include"
BUILD_DIR = SRC_ROOT / "_build"
LIB_DIR = PKG_DIR / "lib"
LIB_PATH = LIB_DIR / "libphmoe.so"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-O2",
              "--expt-relaxed-constexpr"]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libphmoe.so")


def _sources():
    return sorted(CSRC.glob("*.cu"))


def _headers():
    return sorted(list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INCLUDE.glob("*.h")))


def _stale(target: Path, deps) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build(verbose: bool = False, jobs: int | None = None) -> Path:
    nvcc = _nvcc()
    BUILD_DIR.mkdir(parents=True, exist_ok=True)
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    headers = _headers()
    objs = []
    todo = []
    for src in _sources():
        obj = BUILD_DIR / (src.stem + ".o")
        objs.append(obj)
        if _stale(obj, [src, *headers]):
            cmd = [nvcc, *ARCH_FLAGS, *NVCC_FLAGS, "-I", str(INCLUDE), "-c", str(src), "-o", str(obj)]
            todo.append(cmd)

    def run(cmd):
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed ({r.returncode}):\n{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
        return r

    if todo:
        with ThreadPoolExecutor(max_workers=jobs or min(8, os.cpu_count() or 4)) as ex:
            list(ex.map(run, todo))
    if todo or _stale(LIB_PATH, objs):
        link = [nvcc, *ARCH_FLAGS, "-shared", "-o", str(LIB_PATH), *map(str, objs), "--cudart", "static"]
        run(link)
    return LIB_PATH


if __name__ == "__main__":
    p = build(verbose="-v" in sys.argv)
    print(p)
