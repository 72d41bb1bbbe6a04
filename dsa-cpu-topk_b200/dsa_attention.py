"""DeepSeek Sparse Attention forward on B200 — drop-in for the reference module.

Same public names, signatures and layouts as the reference's dsa_attention.py
(Infatoshi/dsa-cpu-topk):

    dsa_attention_triton(q_idx, k_idx, w_idx, Q, K, V, top_k, BLOCK_S=32)          :196-227
    sparse_attention_with_threshold_triton(scores, threshold, Q, K, V)              :298-324
    dsa_attention_split_triton(q_idx, k_idx, w_idx, Q, K, V, top_k, BLOCK_T=32, BLOCK_S=32) :327-344

    q_idx [B,T,HI,DI]  k_idx [B,T,DI]  w_idx [B,T,HI]  Q/K [B,T,HQ,DQ]  V [B,T,HQ,DV]
    -> O [B,T,HQ,DV] float32

Semantics (dsa_attention.py:41-51): scores from the Lightning Indexer,
threshold = k-th largest score of the row (k_eff = min(top_k, T)), keep every
causal key with score >= threshold (ties kept), softmax(Q.K / sqrt(DQ)) over
the kept keys, times V.

Both reference entry points (the fused single kernel and the split
pipeline) give the same result, so both run the same three-stage CUDA
pipeline of libdsa_b200.so: tensor-core indexer -> radix-select top-K (kept
set as a bitmap, or as index lists) -> masked flash attention on the tensor
cores (bf16/fp16, head size 64/128) or a gather attention with an fp32
online softmax.  The reference's
power-of-two and T <= ~512 limits are lifted; its other assertions
(shapes, top_k <= T) are kept.  BLOCK_* arguments are accepted and ignored.
"""
from __future__ import annotations

import math
import os

import torch

import _native


def _check_shapes(q_idx, k_idx, w_idx, Q, K, V):
    assert q_idx.dim() == 4 and Q.dim() == 4 and K.dim() == 4 and V.dim() == 4
    B, T, HQ, DQ = Q.shape
    HI, DI = q_idx.shape[2], q_idx.shape[3]
    assert q_idx.shape[:2] == (B, T) and k_idx.shape == (B, T, DI) and w_idx.shape == (B, T, HI)
    assert K.shape == (B, T, HQ, DQ) and V.shape[:3] == (B, T, HQ)
    assert all(t.is_cuda for t in (q_idx, k_idx, w_idx, Q, K, V)), "inputs must be CUDA tensors"


def dsa_forward(q_idx, k_idx, w_idx, Q, K, V, top_k: int, *, q_row0: int = 0, row_bstep: int = 0,
                workspace: torch.Tensor | None = None) -> torch.Tensor:
    """Whole DSA forward for query rows q_row0..q_row0+T_q-1 of each batch.

    q_idx [B,T_q,HI,DI], w_idx [B,T_q,HI], Q [B,T_q,HQ,DQ] hold those rows;
    k_idx [B,T_k,DI], K [B,T_k,HQ,DQ], V [B,T_k,HQ,DV] hold keys 0..T_k-1.
    Inputs may be strided views (e.g. K/V sliced from a fused projection):
    they are passed to the C ABI as they are when their innermost dimension
    is contiguous and their strides are multiples of 16 bytes.

    Row blocks of one sequence: with ``row_bstep`` != 0, batch b of the
    query-side tensors holds rows q_row0 + b*row_bstep + i, and the key-side
    tensors may have batch size 1 (shared by every block, no copy).  This is
    how a GPU runs its two zig-zag row blocks in one launch per stage.

    ``workspace`` (uint8 CUDA tensor of forward_workspace_bytes(...) bytes) is
    allocated when not given.  Returns O [B,T_q,HQ,DV] float32.
    """
    B, T_q = Q.shape[:2]
    T_k = K.shape[1]
    k_idx = k_idx.to(q_idx.dtype) if k_idx.dtype != q_idx.dtype else k_idx
    K = K.to(Q.dtype) if K.dtype != Q.dtype else K
    V = V.to(Q.dtype) if V.dtype != Q.dtype else V
    w_idx = w_idx if w_idx.dtype == torch.float32 else w_idx.float()
    # key side shared by every batch (row blocks of one sequence): batch stride 0
    if B > 1:
        k_idx, K, V = (t.expand(B, *t.shape[1:]) if t.shape[0] == 1 else t for t in (k_idx, K, V))
    q_idx, k_idx, w_idx, Q, K, V = (_native.prep_strided(t) for t in (q_idx, k_idx, w_idx, Q, K, V))
    O = torch.empty((B, T_q, Q.shape[2], V.shape[3]), device=Q.device, dtype=torch.float32)
    need = _native.forward_workspace_bytes(B, T_q, T_k, top_k, Q.shape[2], V.shape[3], _native.dtype_code(Q))
    if workspace is None or workspace.numel() * workspace.element_size() < need:
        workspace = torch.empty(max(need, 1), device=Q.device, dtype=torch.uint8)
    _native.forward_ex(q_idx, k_idx, w_idx, Q, K, V, O, top_k, workspace, q_row0=q_row0,
                       row_bstep=row_bstep)
    return O


def forward_workspace_bytes(B: int, T_q: int, T_k: int, top_k: int, HQ: int | None = None,
                            DV: int | None = None, dtype: torch.dtype | None = None) -> int:
    """Workspace bytes of dsa_forward; pass the head shape and Q/K/V dtype to size
    the room for the fp16 copy of V (bf16 inputs) as well."""
    if HQ is None:
        return _native.forward_workspace_bytes(B, T_q, T_k, top_k)
    return _native.forward_workspace_bytes(B, T_q, T_k, top_k, HQ, DV, _native._DTYPES[dtype])


def dsa_attention_triton(q_idx, k_idx, w_idx, Q, K, V, top_k: int,
                         BLOCK_S: int = 32) -> torch.Tensor:
    _check_shapes(q_idx, k_idx, w_idx, Q, K, V)
    assert top_k > 0 and top_k <= Q.shape[1], "top_k must be in [1, T]"
    return dsa_forward(q_idx, k_idx, w_idx, Q, K, V, top_k)


def dsa_attention_split_triton(q_idx, k_idx, w_idx, Q, K, V, top_k: int,
                               BLOCK_T: int = 32, BLOCK_S: int = 32) -> torch.Tensor:
    _check_shapes(q_idx, k_idx, w_idx, Q, K, V)
    assert top_k > 0 and top_k <= Q.shape[1], "top_k must be in [1, T]"
    return dsa_forward(q_idx, k_idx, w_idx, Q, K, V, top_k)


def sparse_attention_with_threshold_triton(scores, threshold, Q, K, V) -> torch.Tensor:
    """Attention over keys s <= t with scores[b,t,s] >= threshold[b,t] (dsa_attention.py:298-324)."""
    B, T, _ = scores.shape
    HQ, DQ = Q.shape[-2], Q.shape[-1]
    DV = V.shape[-1]
    assert Q.shape[:2] == (B, T) and K.shape[:2] == (B, T) and V.shape[:2] == (B, T)
    assert threshold.numel() == B * T
    K = K.to(Q.dtype) if K.dtype != Q.dtype else K
    V = V.to(Q.dtype) if V.dtype != Q.dtype else V
    scores = _native.prep(scores.float())
    threshold = _native.prep(threshold.float())
    Q, K, V = (_native.prep_strided(t) for t in (Q, K, V))
    if _native.attn_tc_supported(Q, V) and os.environ.get("DSA_ATTN_GATHER") != "1":
        # tensor cores: the kept set as a bitmap, then the masked flash attention
        return sparse_attention_with_bitmap(kept_bitmap(scores, threshold), Q, K, V)
    out = torch.empty(B, T, HQ, DV, device=Q.device, dtype=torch.float32)
    _native.sparse_attn_ex(None, None, 0, scores, threshold, Q, K, V, out, scale=1.0 / math.sqrt(DQ))
    return out


def kept_bitmap(scores, threshold, *, q_row0: int = 0) -> torch.Tensor:
    """Kept set of each query row as bits: [B*T_q, dsa_bitmap_words(T_k)] int32.

    Bit s % 32 of word s // 32 of row b*T_q + i is set iff s <= q_row0 + i and
    scores[b, i, s] >= threshold[b, i] (the mask of dsa_attention.py:262-266).
    """
    B, T_q, T_k = scores.shape
    scores = _native.prep(scores.float())
    threshold = _native.prep(threshold.float())
    bits = torch.empty(B * T_q, _native.bitmap_words(T_k), device=scores.device, dtype=torch.int32)
    _native.kept_bitmap(scores, threshold, bits, q_row0=q_row0)
    return bits


def sparse_attention_with_bitmap(bits, Q, K, V, *, q_row0: int = 0) -> torch.Tensor:
    """Attention over the set bits of kept_bitmap, on the tensor cores (bf16/fp16, D in {64, 128})."""
    B, T_q, HQ, DQ = Q.shape
    DV = V.shape[-1]
    Q, K, V = (_native.prep_strided(t) for t in (Q, K, V))
    out = torch.empty(B, T_q, HQ, DV, device=Q.device, dtype=torch.float32)
    # workspace: the block summary (skipped key blocks) and, for bf16, the fp16
    # copy of V through which the softmax weights enter P.V in fp16
    nws = _native.sparse_attn_bitmap_workspace_bytes(B, T_q, K.shape[1], HQ, DV, _native.dtype_code(Q))
    ws = torch.empty(nws, device=Q.device, dtype=torch.uint8) if nws else None
    _native.sparse_attn_bitmap_ex(_native.prep(bits), Q, K, V, out, q_row0=q_row0,
                                  scale=1.0 / math.sqrt(DQ), workspace=ws)
    return out


def sparse_attention_with_lists(idx, cnt, idx_cap, scores, threshold, Q, K, V, *,
                                q_row0: int = 0) -> torch.Tensor:
    """Attention over the kept-index lists of topk.topk_select (list form of stage 3).

    Rows whose cnt exceeds idx_cap are recomputed from scores/threshold, so
    those must be given unless idx_cap covers every row.
    """
    B, T_q, HQ, DQ = Q.shape
    DV = V.shape[-1]
    Q, K, V = (_native.prep_strided(t) for t in (Q, K, V))
    out = torch.empty(B, T_q, HQ, DV, device=Q.device, dtype=torch.float32)
    _native.sparse_attn_ex(_native.prep(idx), _native.prep(cnt), idx_cap,
                           None if scores is None else _native.prep(scores.float()),
                           None if threshold is None else _native.prep(threshold.float()),
                           Q, K, V, out, q_row0=q_row0, scale=1.0 / math.sqrt(DQ))
    return out
