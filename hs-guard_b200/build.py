"""Build libhsg.so (all CUDA kernels + the C ABI of include/hsg.h) in-tree for sm_100a with nvcc, and the host
fast-path module _hsg_host (csrc/hsg_host.c, CPython C API) with the C compiler.

    python -m hs_guard_b200.build [--force] [--verbose]

Both are written next to this file so they travel with the source tree; the library links the CUDA runtime
statically and resolves the driver's tensor-map encoder at run time, so it needs no libcuda at link time.
"""
from __future__ import annotations

import importlib
import os
import shutil
import subprocess
import sys
import sysconfig

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
LIB = os.path.join(HERE, "libhsg.so")
SOURCES = [os.path.join(HERE, "csrc", f) for f in sorted(os.listdir(os.path.join(HERE, "csrc")))
           if f.endswith((".cu", ".cuh"))]
MAIN = os.path.join(HERE, "csrc", "hsg_api.cu")
FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-lineinfo", "-O3", "-std=c++17", "-shared",
         "-Xcompiler", "-fPIC", "-I" + os.path.join(ROOT, "include")]
HOST_SRC = os.path.join(HERE, "csrc", "hsg_host.c")
HOST_LIB = os.path.join(HERE, "_hsg_host" + sysconfig.get_config_var("EXT_SUFFIX"))


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


def build_host(force=False):
    """Compile the _hsg_host extension module when it is missing or older than its source."""
    if not force and os.path.exists(HOST_LIB) and os.path.getmtime(HOST_LIB) >= os.path.getmtime(HOST_SRC):
        return HOST_LIB
    cc = os.environ.get("CC") or shutil.which("gcc") or shutil.which("cc")
    if not cc:
        raise RuntimeError("no C compiler for " + HOST_SRC)
    tmp = "%s.%d.tmp" % (HOST_LIB, os.getpid())  # ranks that build at once do not share a temporary
    cmd = [cc, "-O2", "-shared", "-fPIC", "-Wall", "-I" + sysconfig.get_paths()["include"], "-o", tmp, HOST_SRC]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError("building _hsg_host failed:\n" + res.stdout + res.stderr)
    os.replace(tmp, HOST_LIB)
    return HOST_LIB


_HOST = None


def host():
    """The _hsg_host module (built first if needed); raises if it cannot be built or loaded."""
    global _HOST
    if _HOST is None:
        build_host()
        _HOST = importlib.import_module("hs_guard_b200._hsg_host")
    return _HOST


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="--verbose" in sys.argv)
    build_host(force="--force" in sys.argv)
    print(LIB)
    print(HOST_LIB)
