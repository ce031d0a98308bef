"""Build ``libs8b.so`` (all kernels + the C ABI) for sm_100a, in-tree.

    python -m superl8_serve_b200.csrc.build [--force] [--verbose]

Each ``.cu`` compiles to an object under ``_build/`` in parallel, then one shared library is
linked next to the package (``superl8_serve_b200/libs8b.so``). Objects are rebuilt when a
source or header is newer. Extra nvcc flags: ``S8B_NVCC_FLAGS``.
"""

from __future__ import annotations

import os
import shlex
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

CSRC = Path(__file__).resolve().parent
PKG = CSRC.parent
REPO = PKG.parent
BUILD = REPO / "_build"
LIB = PKG / "libs8b.so"
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O3", "--expt-relaxed-constexpr",
         "-I", str(REPO / "include")]


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted((REPO / "include").glob("*.h"))


def _run(cmd: list[str], verbose: bool) -> None:
    if verbose:
        print(" ".join(shlex.quote(c) for c in cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed ({r.returncode}):\n{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    if verbose and (r.stdout or r.stderr):
        print(r.stdout, r.stderr, sep="\n")


def build(force: bool = False, verbose: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    extra = shlex.split(os.environ.get("S8B_NVCC_FLAGS", ""))
    hdr_mtime = max((h.stat().st_mtime for h in headers()), default=0.0)
    objs, jobs = [], []
    for src in sources():
        obj = BUILD / (src.stem + ".o")
        objs.append(obj)
        stale = (force or not obj.exists() or obj.stat().st_mtime < src.stat().st_mtime
                 or obj.stat().st_mtime < hdr_mtime)
        if stale:
            jobs.append([NVCC, *ARCH, *FLAGS, *extra, "-c", str(src), "-o", str(obj)])
    if jobs:
        with ThreadPoolExecutor(max_workers=min(len(jobs), os.cpu_count() or 4)) as ex:
            list(ex.map(lambda c: _run(c, verbose), jobs))
    newest = max(o.stat().st_mtime for o in objs)
    if force or jobs or not LIB.exists() or LIB.stat().st_mtime < newest:
        tmp = LIB.with_suffix(".so.tmp")
        _run([NVCC, *ARCH, "-shared", "-o", str(tmp), *map(str, objs), "-lcudart"], verbose)
        os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    p = build(force="--force" in sys.argv, verbose="--verbose" in sys.argv)
    print(p)
