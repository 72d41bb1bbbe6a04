"""GPU: Lightning Indexer scores (stage 1) against the oracle / golden fixtures.

Tolerance: fp32 inputs rtol 1e-3 (atol 1e-4 as in test_indexer.py:20-21);
bf16 inputs rtol 2e-2 — both stated by the north-star parity bar."""
import glob
import math
import os

import pytest
import torch

from conftest import GOLDEN, golden, t
import dsa_oracle as o

pytestmark = pytest.mark.gpu


def close(out, ref, rtol, atol):
    fin = torch.isfinite(ref)
    assert torch.equal(torch.isfinite(out), fin), "mask pattern differs"
    assert torch.isneginf(out[~fin]).all()
    err = (out[fin] - ref[fin]).abs()
    assert bool((err <= atol + rtol * ref[fin].abs()).all()), f"max err {err.max().item()}"


@pytest.mark.parametrize("name", sorted(os.path.basename(p)[:-4] for p in glob.glob(os.path.join(GOLDEN, "indexer_*.npz"))))
def test_scores_match_golden(cuda, name):
    from lightning_indexer import indexer_scores_triton, topk_mask
    d = golden(name)
    out = indexer_scores_triton(t(d["q"], cuda), t(d["k"], cuda), t(d["w"], cuda), BLOCK_T=32, BLOCK_S=32)
    close(out.cpu(), t(d["scores"]), 1e-3, 1e-4)
    # which -inf positions torch.topk picks in rows with fewer than k causal
    # entries is unspecified, so agreement is measured on causal entries
    T = out.shape[-1]
    causal = torch.ones(T, T, dtype=torch.bool).tril()
    agree = (topk_mask(out, 8).cpu() == t(d["mask8"]))[:, causal].float().mean().item()
    assert agree > 0.99
    assert (topk_mask(out, 8).sum(-1) == 8).all()


def test_projection_pipeline_matches_golden(cuda):
    from lightning_indexer import indexer_triton
    d = golden("project")
    out = indexer_triton(*(t(d[n], cuda) for n in ("h", "W_Q", "W_K", "W_W")), int(d["H"]), int(d["d"]))
    ref = t(d["scores"])
    fin = torch.isfinite(ref)
    assert (out.cpu()[fin] - ref[fin]).abs().max() < 1e-3


@pytest.mark.parametrize("B,T,HI,DI,dtype", [
    (16, 512, 4, 32, torch.float32),      # config c1 shapes
    (2, 333, 3, 48, torch.float32),       # ragged: non-power-of-2 T, HI, DI
    (1, 1, 4, 32, torch.float32),         # single row
    (1, 700, 8, 64, torch.bfloat16),
    (1, 1024, 16, 128, torch.bfloat16),
    (2, 257, 4, 16, torch.float16),
])
def test_scores_random(cuda, B, T, HI, DI, dtype):
    from lightning_indexer import indexer_scores
    qi, ki, wi, *_ = o.make_inputs(B, T, HI, DI, 1, 16, 16, dtype=dtype)
    out = indexer_scores(qi.to(cuda), ki.to(cuda), wi.to(cuda)).cpu()
    ref = o.indexer_scores(qi, ki, wi)
    rtol = 1e-3 if dtype == torch.float32 else 2e-2
    # atol covers cancellation in the w-weighted sum, relative to its terms' size
    atol = rtol * math.sqrt(DI) * 0.1
    close(out, ref, rtol, atol)


def test_row_offset_and_fill(cuda):
    from lightning_indexer import indexer_scores
    qi, ki, wi, *_ = o.make_inputs(2, 300, 4, 32, 1, 16, 16)
    full = o.indexer_scores(qi, ki, wi)
    out = indexer_scores(qi[:, 100:230].to(cuda), ki.to(cuda), wi[:, 100:230].to(cuda), q_row0=100).cpu()
    close(out, full[:, 100:230], 1e-3, 1e-4)
    # without fill_upper the causal part is still exact
    out2 = indexer_scores(qi.to(cuda), ki.to(cuda), wi.to(cuda), fill_upper=False).cpu()
    causal = torch.ones(300, 300, dtype=torch.bool).tril()
    assert torch.allclose(out2[:, causal], full[:, causal], rtol=1e-3, atol=1e-4)


@pytest.mark.parametrize("B,T,HI,DI,dtype", [(4, 512, 4, 32, torch.float32), (2, 333, 3, 48, torch.float32),
                                             (1, 200, 8, 32, torch.bfloat16), (2, 130, 2, 7, torch.float32)])
def test_small_head_simt_kernel_bitwise(cuda, B, T, HI, DI, dtype, monkeypatch):
    """The staged-once kernel for small heads gives the same fp32 bits as the
    generic CUDA-core kernel (same products, same summation order)."""
    from lightning_indexer import indexer_scores
    qi, ki, wi, *_ = (x.to(cuda) for x in o.make_inputs(B, T, HI, DI, 1, 16, 16, dtype=dtype))
    monkeypatch.setenv("DSA_FORCE_SIMT_INDEXER", "1")
    small = indexer_scores(qi, ki, wi)
    monkeypatch.setenv("DSA_INDEXER_SIMT_GENERIC", "1")
    generic = indexer_scores(qi, ki, wi)
    assert torch.equal(small, generic)


@pytest.mark.parametrize("dtype,HI,DI,dm", [(torch.float32, 4, 32, 96), (torch.bfloat16, 16, 128, 256)])
def test_concatenated_projection_matches_separate_matmuls(cuda, dtype, HI, DI, dm, monkeypatch):
    """project() as one GEMM over [W_Q | W_K | W_W] with strided q/k/w views
    gives the scores of the reference's three matmuls (lightning_indexer.py:36-42)."""
    from lightning_indexer import indexer_triton, project
    g = torch.Generator().manual_seed(HI + DI)
    B, T = 2, 384
    h = torch.randn(B, T, dm, generator=g).to(dtype).to(cuda)
    W = [(torch.randn(dm, n, generator=g) / dm ** 0.5).to(dtype).to(cuda) for n in (HI * DI, DI, HI)]
    q, k, w = project(h, *W, HI, DI)
    assert not q.is_contiguous() and not k.is_contiguous()
    fused = indexer_triton(h, *W, HI, DI)
    monkeypatch.setenv("DSA_PROJECT_SEPARATE", "1")
    sep = indexer_triton(h, *W, HI, DI)
    fin = torch.isfinite(sep)
    tol = 1e-4 if dtype == torch.float32 else 2e-2
    err = (fused[fin] - sep[fin]).abs()
    assert bool((err <= tol * sep[fin].abs() + tol * sep[fin].abs().mean()).all()), err.max().item()
