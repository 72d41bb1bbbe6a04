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
    """build.py compiles every CUDA source for sm_100a only."""
    import build
    assert build.ARCH == ["-gencode", "arch=compute_100a,code=sm_100a"]


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


def test_bitmap_entry_points_validate_on_the_host(lib):
    """Word counts, sizes and dtypes of the bitmap path are checked before any
    device work (fake non-null pointers are never dereferenced)."""
    import _native
    for T, w in [(1, 4), (128, 4), (129, 8), (512, 16), (32768, 1024)]:
        assert lib.dsa_bitmap_words(T) == w
    # the forward workspace holds the bitmap beside scores, thresholds and lists
    assert lib.dsa_forward_workspace_bytes(1, 1024, 1024, 64) >= 1024 * 1024 * 4 + 1024 * 32 * 4
    fake = ctypes.c_void_p(256)
    # too few words per row
    rc = lib.dsa_kept_bitmap(fake, fake, fake, 1, 128, 1024, 0, 8, None)
    assert rc == _native.DSA_ERR_INVALID and b"words_per_row" in lib.dsa_last_error_string()
    rc = lib.dsa_topk_select_bitmap(fake, 128, 1024, 128, 0, 1, 16, fake, None, None, 32, None)
    assert rc == _native.DSA_ERR_INVALID
    rc = lib.dsa_topk_select_bitmap(fake, 128, 1024, 128, 0, 1, 16, fake, None, fake, 30, None)
    assert rc == _native.DSA_ERR_INVALID
    # fp32 attention inputs are not a tensor-core case
    rc = lib.dsa_sparse_attn_bitmap(fake, 32, fake, fake, fake, fake, 1, 128, 1024, 0, 4, 128, 128,
                                    ctypes.c_float(0.1), _native.DSA_F32, None)
    assert rc == _native.DSA_ERR_UNSUPPORTED
    rc = lib.dsa_sparse_attn_bitmap(None, 32, fake, fake, fake, fake, 1, 128, 1024, 0, 4, 128, 128,
                                    ctypes.c_float(0.1), _native.DSA_BF16, None)
    assert rc == _native.DSA_ERR_INVALID


def test_checked_library_exports_every_declared_symbol():
    """libdsa_b200_checked.so (index checks that flag instead of faulting) has the same boundary."""
    import build
    path = build.build(checked=True)
    out = subprocess.run(["nm", "-D", "--defined-only", path], capture_output=True, text=True, check=True).stdout
    exported = set(re.findall(r" T (dsa_\w+)", out))
    missing = [n for n in declared() if n not in exported]
    assert not missing, missing
