"""Shared test set-up: import paths, the `gpu` marker, golden-fixture loader."""
import os
import sys

import numpy as np
import pytest
import torch

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(REPO, "dsa-cpu-topk_b200")
ORACLE = os.path.join(REPO, "oracle")
GOLDEN = os.path.join(REPO, "tests", "golden")
for p in (PKG, ORACLE):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and libdsa_b200.so")


def golden(name):
    d = np.load(os.path.join(GOLDEN, name + ".npz"))
    return {k: d[k] for k in d.files}


def t(a, device="cpu", dtype=None):
    x = torch.from_numpy(np.asarray(a))
    if dtype is not None:
        x = x.to(dtype)
    return x.to(device)


@pytest.fixture(scope="session")
def cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")


# The north star's bf16/fp16 parity bar for attention outputs: rtol 2e-2,
# elementwise.  ATOL_16 is the absolute floor for outputs near zero (an output
# that averages thousands of kept V rows can be ~1e-3 by cancellation).
RTOL_16, ATOL_16 = 2e-2, 1e-3


def assert_close_elementwise(out, ref, *, rtol=RTOL_16, atol=ATOL_16, what="output"):
    """|out - ref| <= atol + rtol*|ref| for every element; prints and returns the
    largest error relative to max(|ref|, atol)."""
    out = out.detach().float().cpu()
    ref = ref.detach().float().cpu()
    assert out.shape == ref.shape, (out.shape, ref.shape)
    err = (out - ref).abs()
    rel = (err / ref.abs().clamp_min(atol)).max().item() if err.numel() else 0.0
    bad = ~(err <= atol + rtol * ref.abs())
    print(f"{what}: max abs err {err.max().item() if err.numel() else 0.0:.3e}, "
          f"max rel err {rel:.3e} (|ref| floored at {atol:g}), bar rtol {rtol:g} atol {atol:g}")
    assert not bool(bad.any()), (f"{what}: {int(bad.sum())} of {bad.numel()} elements outside "
                                 f"rtol {rtol:g} / atol {atol:g}; max rel err {rel:.3e}")
    return rel
