"""Builds libflowedge_b200.so in-tree (nvcc for sm_100a, g++ -std=c++23 for host code).

    python -m flowedge_b200.build [--force]

Objects go to flowedge_b200/_build/ (not committed); the library is written
next to this file so it travels with the source tree.
"""

from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
BUILD = HERE / "_build"
LIB = HERE / "libflowedge_b200.so"
INCLUDE = HERE.parent / "include"

NVCC = os.environ.get("NVCC", shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc")
CXX = os.environ.get("CXX", "g++")
CUDA_HOME = Path(NVCC).resolve().parents[1]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++20", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
              "--expt-relaxed-constexpr", "-I", str(CSRC), "-I", str(INCLUDE)] + ARCH
CXX_FLAGS = ["-O2", "-std=c++23", "-fPIC", "-fvisibility=hidden", "-Wall", "-Wextra", "-Wno-unused-parameter",
             "-I", str(CSRC), "-I", str(INCLUDE), "-I", str(CUDA_HOME / "include")]


def _sources():
    return sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cc"))


def _headers_mtime():
    files = list(CSRC.glob("*.h")) + list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h"))
    return max((f.stat().st_mtime for f in files), default=0.0)


def _compile(src: Path, force: bool) -> Path:
    obj = BUILD / (src.name + ".o")
    if not force and obj.exists() and obj.stat().st_mtime >= max(src.stat().st_mtime, _headers_mtime()):
        return obj
    if src.suffix == ".cu":
        cmd = [NVCC, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
    else:
        cmd = [CXX, *CXX_FLAGS, "-c", str(src), "-o", str(obj)]
    result = subprocess.run(cmd, capture_output=True, text=True)
    if result.returncode != 0:
        raise RuntimeError(f"compile failed: {src.name}\n{' '.join(cmd)}\n{result.stdout}\n{result.stderr}")
    return obj


def build(force: bool = False, verbose: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as pool:
        objs = list(pool.map(lambda s: _compile(s, force), _sources()))
    if force or not LIB.exists() or LIB.stat().st_mtime < max(o.stat().st_mtime for o in objs):
        cmd = [NVCC, "-shared", *ARCH, "-o", str(LIB), *map(str, objs), "-lcuda"]
        result = subprocess.run(cmd, capture_output=True, text=True)
        if result.returncode != 0:
            raise RuntimeError(f"link failed\n{' '.join(cmd)}\n{result.stdout}\n{result.stderr}")
    if verbose:
        print(f"built {LIB}")
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
