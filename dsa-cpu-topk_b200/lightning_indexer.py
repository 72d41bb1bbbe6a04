"""DeepSeek-V3.2 Lightning Indexer on B200 — drop-in for the reference module.

Same public names, signatures and tensor layouts as the reference's
lightning_indexer.py (Infatoshi/dsa-cpu-topk):

    I[b, t, s] = sum_j w[b, t, j] * ReLU(<q[b, t, j, :], k[b, s, :]>)   for s <= t, else -inf

    project(h, W_Q, W_K, W_W, num_heads, head_dim)        lightning_indexer.py:36-42
    indexer_scores_triton(q, k, w, BLOCK_T=64, BLOCK_S=64) lightning_indexer.py:100-125
    indexer_triton(h, W_Q, W_K, W_W, num_heads, head_dim)  lightning_indexer.py:128-130
    topk_mask(scores, k)                                   lightning_indexer.py:137-144

The ``*_triton`` names are kept so callers switch by import path only; there
is no Triton here.  The scores come from libdsa_b200.so (stage 1:
tcgen05 tensor cores for bf16, IEEE-fp32 CUDA cores for fp32).  Unlike the
reference, head_dim need not be a power of two and T is unrestricted.
BLOCK_T / BLOCK_S are accepted for compatibility and ignored (the kernels
pick their own tiles).

The reference's pure-torch variants (indexer_scores_torch, indexer_torch)
are its CPU/oracle path; they are not part of this GPU package.
"""
from __future__ import annotations

import os

import torch

import _native
from topk import topk_select


_W_CAT: dict = {}


def _concat_weights(W_Q, W_K, W_W):
    """[W_Q | W_K | W_W] along the output dimension, cached while the three
    weight tensors are unchanged (same storage and version counter)."""
    key = tuple((w.data_ptr(), w._version, tuple(w.shape), w.dtype) for w in (W_Q, W_K, W_W))
    hit = _W_CAT.get(key)
    if hit is None:
        _W_CAT.clear()
        hit = torch.cat([W_Q, W_K, W_W], dim=1).contiguous()
        _W_CAT[key] = hit
    return hit


def project(h: torch.Tensor, W_Q: torch.Tensor, W_K: torch.Tensor, W_W: torch.Tensor,
            num_heads: int, head_dim: int):
    """h @ W_Q / W_K / W_W (lightning_indexer.py:36-42) as ONE cuBLAS GEMM over the
    concatenated weights; q, k and w are strided views of its output, which the
    indexer reads in place (no copies).  DSA_PROJECT_SEPARATE=1 runs the three
    matmuls of the reference instead."""
    B, T, _ = h.shape
    if os.environ.get("DSA_PROJECT_SEPARATE") == "1" or not (W_Q.dtype == W_K.dtype == W_W.dtype):
        return (h @ W_Q).view(B, T, num_heads, head_dim), h @ W_K, h @ W_W
    HD = num_heads * head_dim
    out = h @ _concat_weights(W_Q, W_K, W_W)
    q = out[..., :HD].view(B, T, num_heads, head_dim)
    k = out[..., HD:HD + head_dim]
    w = out[..., HD + head_dim:]
    return q, k, w


def indexer_scores_triton(q: torch.Tensor, k: torch.Tensor, w: torch.Tensor,
                          BLOCK_T: int = 64, BLOCK_S: int = 64) -> torch.Tensor:
    """q: [B,T,H,d]  k: [B,T,d]  w: [B,T,H]  ->  scores [B,T,T] fp32 (off-causal = -inf)."""
    assert q.is_cuda and k.is_cuda and w.is_cuda
    B, T, H, d = q.shape
    assert k.shape == (B, T, d)
    assert w.shape == (B, T, H)
    return indexer_scores(q, k, w)


def indexer_scores(q: torch.Tensor, k: torch.Tensor, w: torch.Tensor, *, q_row0: int = 0,
                   row_bstep: int = 0, fill_upper: bool = True) -> torch.Tensor:
    """Scores of query rows q_row0 + b*row_bstep + i (i < T_q) against keys 0..T_k-1.

    q: [B,T_q,H,d], k: [B,T_k,d] (or [1,T_k,d], shared), w: [B,T_q,H] -> [B,T_q,T_k]
    fp32.  Strided views are read in place.
    """
    assert q.dim() == 4 and k.dim() == 3 and w.dim() == 3
    B, T_q, H, d = q.shape
    assert k.shape[0] in (B, 1) and k.shape[2] == d and w.shape == (B, T_q, H)
    if k.dtype != q.dtype:
        k = k.to(q.dtype)
    if k.shape[0] != B:
        k = k.expand(B, *k.shape[1:])
    w = w if w.dtype == torch.float32 else w.float()
    q, k, w = _native.prep_strided(q), _native.prep_strided(k), _native.prep_strided(w)
    scores = torch.empty((B, T_q, k.shape[1]), device=q.device, dtype=torch.float32)
    _native.indexer_scores_ex(q, k, w, scores, q_row0=q_row0, row_bstep=row_bstep,
                              fill_upper=fill_upper)
    return scores


def indexer_triton(h, W_Q, W_K, W_W, num_heads, head_dim, **kw):
    q, k, w = project(h, W_Q, W_K, W_W, num_heads, head_dim)
    return indexer_scores_triton(q, k, w, **kw)


def topk_mask(scores: torch.Tensor, k: int) -> torch.Tensor:
    """Boolean mask of exactly min(k, T) key positions per query row.

    Like the reference (lightning_indexer.py:137-144) it marks k positions, not
    all ties: every position above the k-th largest value, then positions equal
    to it in ascending order until k are marked (torch.topk leaves the choice
    among equal values unspecified).
    """
    B, T, N = scores.shape
    k_eff = min(k, N)
    s = _native.prep(scores.float())
    thr, _, _ = topk_select(s, k_eff, return_idx=False)
    thr = thr.view(B, T, 1)
    gt = s > thr
    eq = s == thr
    need = k_eff - gt.sum(-1, keepdim=True)
    return gt | (eq & (eq.cumsum(-1) <= need))


def quantize_fp8(x: torch.Tensor):
    """Per-row e4m3 quantisation of x's last dimension: (x8, scale) with
    x ~= x8.float() * scale[..., None], scale = max|row| / 448."""
    x = x.contiguous()
    x8 = torch.empty(x.shape, device=x.device, dtype=torch.float8_e4m3fn)
    scale = torch.empty(x.shape[:-1], device=x.device, dtype=torch.float32)
    _native.quantize_fp8_rows(x, x8, scale)
    return x8, scale


def indexer_scores_fp8(q: torch.Tensor, k: torch.Tensor, w: torch.Tensor, *, q_row0: int = 0,
                       fill_upper: bool = True) -> torch.Tensor:
    """The FP8 Lightning Indexer: q [B,T_q,H,d] and k [B,T_k,d] (any float type) are
    quantised to e4m3 per row; the key scales multiply the score columns and the
    query scales fold into w.  Same output as indexer_scores up to e4m3 rounding."""
    q8, q_s = quantize_fp8(q)
    k8, k_s = quantize_fp8(k)
    w2 = (w.float() * q_s).contiguous()
    B, T_q = q.shape[:2]
    scores = torch.empty((B, T_q, k.shape[1]), device=q.device, dtype=torch.float32)
    _native.indexer_scores_fp8(q8, k8, w2, k_s.contiguous(), scores, q_row0=q_row0, fill_upper=fill_upper)
    return scores
