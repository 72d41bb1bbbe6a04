"""TEST INFRASTRUCTURE ONLY: compile the reference's own AVX-512 top-K.

Builds `topk_avx512.cpp` of Infatoshi/dsa-cpu-topk, read in place from the
reference checkout (never copied into this repository), into
``oracle/_ref/topk_avx512_ref*.so``.  The reference builds the same file with
``torch.utils.cpp_extension.load`` (dsa_hybrid.py:22-33, bench_avx512.py:12-23);
this recipe uses the same tool and flags, with two changes so the binary runs
on any AVX-512 host the GPU box may have:

  * ``-march=x86-64-v4`` (AVX-512 F/BW/CD/DQ/VL) instead of ``-march=native``;
  * no ``-mavx512vbmi/-mavx512vbmi2`` (the source uses only AVX-512F
    intrinsics, topk_avx512.cpp:44-49, so these only widen what the compiler
    may emit).

``-O3 -fopenmp -funroll-loops -ffast-math`` are kept as in the reference.
``/usr/bin/g++`` is used because the image's default ``g++`` cannot link
``-fopenmp``.

Usage:  python oracle/build_ref.py [REFERENCE_DIR]
The resulting module is loaded by :func:`load_ref` (tests and bench only).
"""
from __future__ import annotations

import glob
import importlib.machinery
import importlib.util
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REF_OUT = os.path.join(HERE, "_ref")
MOD_NAME = "topk_avx512_ref"
def build(reference_dir: str | None = None, verbose: bool = False) -> str | None:
    """Compile the reference's topk_avx512.cpp found in ``reference_dir`` (or
    $DSA_REFERENCE_DIR); returns the built module's path, or None when neither
    names a directory holding the source."""
    reference_dir = reference_dir or os.environ.get("DSA_REFERENCE_DIR")
    if not reference_dir:
        return None
    src = os.path.join(reference_dir, "topk_avx512.cpp")
    if not os.path.exists(src):
        return None
    import torch  # noqa: F401  (cpp_extension needs torch)
    from torch.utils.cpp_extension import load

    os.makedirs(REF_OUT, exist_ok=True)
    if os.path.exists("/usr/bin/g++"):
        os.environ["CXX"] = "/usr/bin/g++"
        os.environ["CC"] = "/usr/bin/gcc"
    load(
        name=MOD_NAME,
        sources=[src],
        extra_cflags=["-O3", "-fopenmp", "-march=x86-64-v4", "-funroll-loops", "-ffast-math"],
        extra_ldflags=["-fopenmp"],
        build_directory=REF_OUT,
        verbose=verbose,
    )
    return find_so()


def find_so() -> str | None:
    hits = sorted(glob.glob(os.path.join(REF_OUT, MOD_NAME + "*.so")))
    return hits[0] if hits else None


def host_has_avx512() -> bool:
    try:
        with open("/proc/cpuinfo") as f:
            flags = f.read()
    except OSError:
        return False
    return all(x in flags for x in ("avx512f", "avx512bw", "avx512dq", "avx512vl", "avx512cd"))


def load_ref():
    """Import the prebuilt reference top-K module, or return None."""
    so = find_so()
    if so is None or not host_has_avx512():
        return None
    import torch  # noqa: F401
    loader = importlib.machinery.ExtensionFileLoader(MOD_NAME, so)
    spec = importlib.util.spec_from_file_location(MOD_NAME, so, loader=loader)
    mod = importlib.util.module_from_spec(spec)
    loader.exec_module(mod)
    return mod


if __name__ == "__main__":
    out = build(sys.argv[1] if len(sys.argv) > 1 else None, verbose=True)
    print(out or "usage: build_ref.py <reference checkout> (or set DSA_REFERENCE_DIR); nothing built")
