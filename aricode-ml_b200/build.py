"""Compile the CUDA decode library in-tree: aricode-ml_b200/libb2dec.so (sm_100a).

    python aricode-ml_b200/build.py [--verbose]

nvcc cross-compiles without a GPU; the resulting .so is what the ctypes host
loop (runtime.py) and the tests load.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
LIB = PKG / "libb2dec.so"
SOURCES = ["runtime.cu", "capi.cu", "noalloc.cu"]
HEADERS = ["b2_common.cuh", "gemv.cuh", "attn.cuh", "kernels.cuh", "token.cuh", "json.h"]

NVCC_FLAGS = [
    "-O3", "-std=c++17", "-lineinfo",
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-Xcompiler", "-fPIC", "-shared",
    "-Xcompiler", "-Wall",
]


def nvcc():
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def stale():
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    deps = [CSRC / s for s in SOURCES + HEADERS] + [PKG.parent / "include" / "b2dec.h"]
    return any(p.stat().st_mtime > t for p in deps if p.exists())


def build(force=False, verbose=False):
    if not force and not stale():
        return LIB
    cmd = [nvcc(), *NVCC_FLAGS, *(["-Xptxas", "-v"] if verbose else []),
           "-o", str(LIB), *[str(CSRC / s) for s in SOURCES]]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("nvcc failed:\n" + r.stdout + r.stderr)
    if verbose:
        sys.stderr.write(r.stdout + r.stderr)
    return LIB


if __name__ == "__main__":
    build(force=True, verbose="--verbose" in sys.argv)
    print(LIB)
