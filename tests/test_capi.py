"""CPU: the C-ABI library loads, exports every declared symbol, and validates
arguments on the host (no kernel runs here)."""
import ctypes
import os
import re
import subprocess

import pytest

from conftest import REPO, PKG

HEADER = os.path.join(REPO, "include", "dsa_b200.h")


def declared():
    src = open(HEADER).read()
    return sorted(set(re.findall(r"DSA_API\s+[\w\s\*]+?\b(dsa_\w+)\s*\(", src)))


@pytest.fixture(scope="module")
def lib():
    import _native
    if not os.path.exists(_native.LIB_PATH):
        import build
        build.build()
    return _native.lib()


def test_header_declares_the_boundary():
    names = declared()
    for n in ["dsa_indexer_scores", "dsa_topk_select", "dsa_sparse_attn", "dsa_sparse_attn_threshold",
              "dsa_forward", "dsa_forward_workspace_bytes", "dsa_last_error_string", "dsa_version"]:
        assert n in names


def test_library_exports_every_declared_symbol(lib):
    out = subprocess.run(["nm", "-D", "--defined-only", os.path.join(PKG, "libdsa_b200.so")],
                         capture_output=True, text=True, check=True).stdout
    exported = set(re.findall(r" T (dsa_\w+)", out))
    missing = [n for n in declared() if n not in exported]
    assert not missing, missing
    for n in declared():
        getattr(lib, n)


def test_library_is_built_for_sm100a():
    out = subprocess.run(["/usr/local/cuda/bin/cuobjdump", "--list-elf",
                          os.path.join(PKG, "libdsa_b200.so")], capture_output=True, text=True)
    if out.returncode != 0:
        pytest.skip("cuobjdump unavailable")
    assert "sm_100a" in out.stdout


def test_host_validation_errors(lib):
    import _native
    assert lib.dsa_version() >= 1
    # k > row_len is rejected before any device work
    rc = lib.dsa_topk_select(None, 4, 16, 16, 1, 0, 0, 17, None, None, None, 0, None)
    assert rc == _native.DSA_ERR_INVALID
    assert b"k" in lib.dsa_last_error_string()
    rc = lib.dsa_sparse_attn_threshold(None, None, None, None, None, None, 1, 1, 1, 0, 1, 32, 16, 1.0, 0, None)
    assert rc == _native.DSA_ERR_UNSUPPORTED  # DQ != DV
    rc = lib.dsa_indexer_scores(None, None, None, None, 1, 1, 1, 0, 1, 1, 0, 1, None)
    assert rc == _native.DSA_ERR_INVALID
    assert lib.dsa_forward_workspace_bytes(1, 512, 512, 32) > 512 * 512 * 4
    assert lib.dsa_forward_workspace_bytes(1, 512, 512, 0) == 0
    with pytest.raises(AssertionError):
        _native._check(_native.DSA_ERR_INVALID, "x")
    with pytest.raises(RuntimeError):
        _native._check(_native.DSA_ERR_CUDA, "x")
