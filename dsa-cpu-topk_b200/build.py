"""Build libdsa_b200.so in-tree with nvcc for sm_100a.

    python dsa-cpu-topk_b200/build.py [--force] [--checked]

Each .cu file under csrc/ is compiled to an object in csrc/_build/ (only when
its source or a header is newer) and linked into
``dsa-cpu-topk_b200/libdsa_b200.so``.  The library exports only the C ABI of
include/dsa_b200.h; it links the CUDA runtime statically, so it needs no
torch at build or load time.

--checked builds libdsa_b200_checked.so instead (objects in csrc/_build_checked/):
the same sources with -DDSA_DEBUG_CHECKS, whose guarded accesses check their
index and set a device flag (read by dsa_debug_status) instead of accessing.
"""
from __future__ import annotations

import glob
import os
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
OBJ = os.path.join(CSRC, "_build")
LIB = os.path.join(PKG, "libdsa_b200.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-fvisibility=hidden",
         "--expt-relaxed-constexpr", "-I" + os.path.join(REPO, "include")]


def _newest(paths):
    return max((os.path.getmtime(p) for p in paths), default=0.0)


def build(force: bool = False, verbose: bool = False, checked: bool = False) -> str:
    obj_dir = OBJ + "_checked" if checked else OBJ
    lib = LIB[:-3] + "_checked.so" if checked else LIB
    extra = ["-DDSA_DEBUG_CHECKS"] if checked else []
    os.makedirs(obj_dir, exist_ok=True)
    sources = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    headers = glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(REPO, "include", "*.h"))
    hdr_time = _newest(headers)
    objs = []
    for src in sources:
        obj = os.path.join(obj_dir, os.path.basename(src)[:-3] + ".o")
        objs.append(obj)
        if force or not os.path.exists(obj) or os.path.getmtime(obj) < max(os.path.getmtime(src), hdr_time):
            cmd = [NVCC, *ARCH, *FLAGS, *extra, "-c", src, "-o", obj]
            if verbose:
                print(" ".join(cmd), flush=True)
            subprocess.run(cmd, check=True)
    if force or not os.path.exists(lib) or os.path.getmtime(lib) < _newest(objs):
        cmd = [NVCC, *ARCH, "-shared", "-Xcompiler", "-fPIC", "-o", lib, *objs]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    return lib


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True, checked="--checked" in sys.argv))
