"""Builds libaps2026_b200.so in-tree from aps2026_b200/csrc for sm_100a.

Each CUDA translation unit is compiled by nvcc (``-gencode
arch=compute_100a,code=sm_100a -lineinfo -O3``, IEEE division and square
root, no fast-math: the routing quantiser and the LayerNorm need them), the
host C++ by g++, and everything is linked into one shared library next to
this file. Objects go to ``aps2026_b200/_build`` and are rebuilt only when a
source or header is newer.

Run as ``python -m aps2026_b200.build [-v]`` (``-v`` prints ptxas register /
spill / shared-memory use per kernel).
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
BUILD = HERE / "_build"
LIB = HERE / "libaps2026_b200.so"
INCLUDE = HERE.parent / "include"

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
CXX = "/usr/bin/g++" if Path("/usr/bin/g++").exists() else "g++"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", *ARCH, "-Xcompiler", "-fPIC",
              "-Xcompiler", "-O3", "--expt-relaxed-constexpr"]
CXX_FLAGS = ["-O3", "-std=c++17", "-fPIC", "-Wall", "-Wextra", "-march=x86-64-v3"]


def _sources() -> list[Path]:
    return sorted(p for p in CSRC.iterdir() if p.suffix in (".cu", ".cpp"))


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h")) + sorted(INCLUDE.glob("*.cuh"))


def _compile(src: Path, verbose: bool) -> Path:
    obj = BUILD / (src.stem + (".cu.o" if src.suffix == ".cu" else ".cpp.o"))
    newest_dep = max([src.stat().st_mtime] + [h.stat().st_mtime for h in _headers()])
    if obj.exists() and obj.stat().st_mtime >= newest_dep and not verbose:
        return obj
    if src.suffix == ".cu":
        cmd = [NVCC, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
        if verbose:
            cmd[1:1] = ["-Xptxas", "-v"]
    else:
        cmd = [CXX, *CXX_FLAGS, "-c", str(src), "-o", str(obj)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"compile failed: {' '.join(cmd)}\n{res.stdout}\n{res.stderr}")
    if verbose and res.stderr:
        sys.stderr.write(res.stderr)
    return obj


def build(verbose: bool = False) -> Path:
    """Compiles every source (in parallel) and links the shared library."""
    BUILD.mkdir(exist_ok=True)
    srcs = _sources()
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as pool:
        objs = list(pool.map(lambda s: _compile(s, verbose), srcs))
    newest = max(o.stat().st_mtime for o in objs)
    if not LIB.exists() or LIB.stat().st_mtime < newest:
        cmd = [NVCC, "-shared", *ARCH, "-o", str(LIB), *map(str, objs)]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed: {' '.join(cmd)}\n{res.stdout}\n{res.stderr}")
    return LIB


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv[1:]))
