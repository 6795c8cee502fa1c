"""Build libhsg.so (all CUDA kernels + the C ABI of include/hsg.h) in-tree for sm_100a with nvcc.

    python -m hs_guard_b200.build [--force] [--verbose]

The library is written next to this file so it travels with the source tree; it links the CUDA runtime statically
and resolves the driver's tensor-map encoder at run time, so it needs no libcuda at link time.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
LIB = os.path.join(HERE, "libhsg.so")
SOURCES = [os.path.join(HERE, "csrc", f) for f in sorted(os.listdir(os.path.join(HERE, "csrc")))
           if f.endswith((".cu", ".cuh"))]
MAIN = os.path.join(HERE, "csrc", "hsg_api.cu")
FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-lineinfo", "-O3", "-std=c++17", "-shared",
         "-Xcompiler", "-fPIC", "-I" + os.path.join(ROOT, "include")]


def nvcc():
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def stale():
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    return any(os.path.getmtime(s) > t for s in SOURCES + [os.path.join(ROOT, "include", "hsg.h")])


def build(force=False, verbose=False):
    if not force and not stale():
        return LIB
    tmp = LIB + ".tmp"
    cmd = [nvcc()] + FLAGS + (["-Xptxas", "-v"] if verbose else []) + ["-o", tmp, MAIN]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError("nvcc failed:\n" + res.stdout + res.stderr)
    if verbose:
        sys.stderr.write(res.stdout + res.stderr)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="--verbose" in sys.argv)
    print(LIB)
