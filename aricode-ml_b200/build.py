"""Compile the CUDA decode library in-tree: aricode-ml_b200/libb2dec.so (sm_100a).

    python aricode-ml_b200/build.py [--verbose]

nvcc cross-compiles without a GPU; the resulting .so is what the ctypes host
loop (runtime.py) and the tests load. Each .cu file compiles to its own object
(in parallel, into csrc/_obj/, rebuilt only when it or a header is newer), then
one link.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
OBJ = CSRC / "_obj"
LIB = PKG / "libb2dec.so"
FRONT = PKG / "b2run"                    # stdin-tokens front end (host program over the library)
SOURCES = ["runtime.cu", "launch.cu", "token.cu", "prefill.cu", "capi.cu", "noalloc.cu"]
HEADERS = ["b2_common.cuh", "gemv.cuh", "attn.cuh", "kernels.cuh", "token.cuh", "prefill.cuh", "json.h"]

NVCC_FLAGS = [
    "-O3", "-std=c++17", "-lineinfo",
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-Xcompiler", "-fPIC",
    "-Xcompiler", "-Wall",
]


def nvcc():
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def _deps_time():
    deps = [CSRC / h for h in HEADERS] + [PKG.parent / "include" / "b2dec.h"]
    return max(p.stat().st_mtime for p in deps if p.exists())


def _obj(src):
    return OBJ / (Path(src).stem + ".o")


def _stale_obj(src, hdr_t):
    o = _obj(src)
    return not o.exists() or o.stat().st_mtime < max(hdr_t, (CSRC / src).stat().st_mtime)


def stale():
    if not LIB.exists() or not FRONT.exists() or FRONT.stat().st_mtime < (CSRC / "b2run.cpp").stat().st_mtime:
        return True
    hdr_t = _deps_time()
    t = LIB.stat().st_mtime
    return any(_stale_obj(s, hdr_t) or _obj(s).stat().st_mtime > t for s in SOURCES)


def _compile(src, verbose):
    cmd = [nvcc(), *NVCC_FLAGS, *(["-Xptxas", "-v"] if verbose else []), "-c", str(CSRC / src),
           "-o", str(_obj(src))]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src}:\n" + r.stdout + r.stderr)
    return r.stdout + r.stderr


def build(force=False, verbose=False):
    if not force and not stale():
        return LIB
    OBJ.mkdir(exist_ok=True)
    hdr_t = _deps_time()
    todo = [s for s in SOURCES if force or _stale_obj(s, hdr_t)]
    with ThreadPoolExecutor(max_workers=len(todo) or 1) as ex:
        logs = list(ex.map(lambda s: _compile(s, verbose), todo))
    if verbose:
        sys.stderr.write("".join(logs))
    cmd = [nvcc(), "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-o", str(LIB),
           *[str(_obj(s)) for s in SOURCES]]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("nvcc link failed:\n" + r.stdout + r.stderr)
    build_front()
    return LIB


def build_front():
    """The stdin-tokens front end, a host program linked against libb2dec.so."""
    cmd = ["g++", "-O2", "-std=c++17", "-Wall", str(CSRC / "b2run.cpp"), "-o", str(FRONT),
           "-L" + str(PKG), "-lb2dec", "-Wl,-rpath,$ORIGIN"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("g++ failed on b2run.cpp:\n" + r.stdout + r.stderr)
    return FRONT


if __name__ == "__main__":
    build(force=True, verbose="--verbose" in sys.argv)
    print(LIB)
