"""TEST INFRASTRUCTURE ONLY — CPU oracle for the DSA forward hot path.

Only tests/, ``__graft_entry__.smoke()`` and bench.py's ``cpu_baseline`` /
``--impl reference`` legs import this module, and only as the checker or the
timed CPU baseline.  The shipped package never imports it.

It restates, on CPU PyTorch tensors, the reference's own torch variant
(Infatoshi/dsa-cpu-topk):

  * indexer_scores      lightning_indexer.py:26-33  (einsum -> ReLU -> w-sum -> causal -inf)
  * project             lightning_indexer.py:36-42
  * select_threshold    dsa_attention.py:41-46      (k_eff = min(k,T); thr = topk(...)[-1]; keep ties)
  * dsa_attention       dsa_attention.py:35-52      (dense masked softmax over the kept keys)
  * sparse_attention_with_threshold   dsa_attention.py:234-324 (threshold given)
  * topk_mask           lightning_indexer.py:137-144

Everything is computed over query-row chunks with a causal offset so that the
long-context configurations fit in host memory: row t of a chunk sees keys
s <= t exactly as row t of the unchunked einsum does.  bf16 inputs are
upcast to fp32 first (the reference's Triton kernels do the same,
lightning_indexer.py:79,85).

The top-K threshold/index oracle in C (topk_oracle.c) is wrapped by
:func:`topk_select`.
"""
from __future__ import annotations

import ctypes
import math
import os
import subprocess

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(HERE, "_build", "libtopk_oracle.so")
_lib = None


# --------------------------------------------------------------------------
# C top-K oracle
# --------------------------------------------------------------------------

def _load_lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            subprocess.run(["make", "-s", "-C", HERE], check=True)
        lib = ctypes.CDLL(_LIB_PATH)
        i64, f32p, i32p = ctypes.c_int64, ctypes.POINTER(ctypes.c_float), ctypes.POINTER(ctypes.c_int32)
        lib.oracle_topk_select.argtypes = [f32p, i64, i64, i64, i64, i64, ctypes.c_int, i64,
                                           f32p, i32p, i32p, i64]
        lib.oracle_topk_select.restype = ctypes.c_int
        _lib = lib
    return _lib


def topk_select(scores: np.ndarray | torch.Tensor, k: int, *, causal: bool = False,
                rows_per_batch: int | None = None, q_row0: int = 0, idx_cap: int | None = None):
    """Threshold, kept-index lists and counts for every row of ``scores``.

    scores: [..., N] float32 (CPU).  Returns (thr [rows], idx [rows, idx_cap] int32
    padded with -1, cnt [rows] int32).  With ``causal``, row r sits at query
    position q_row0 + r % rows_per_batch and entries s > t count as -inf.
    """
    if isinstance(scores, torch.Tensor):
        scores = scores.detach().cpu().numpy()
    a = np.ascontiguousarray(scores, dtype=np.float32)
    N = a.shape[-1]
    rows = a.size // N if N else 0
    a = a.reshape(rows, N)
    if rows_per_batch is None:
        rows_per_batch = rows if rows else 1
    if idx_cap is None:
        idx_cap = N
    thr = np.empty(rows, np.float32)
    cnt = np.empty(rows, np.int32)
    idx = np.full((rows, idx_cap), -1, np.int32)
    lib = _load_lib()
    f32p, i32p = ctypes.POINTER(ctypes.c_float), ctypes.POINTER(ctypes.c_int32)
    rc = lib.oracle_topk_select(a.ctypes.data_as(f32p), rows, N, N, rows_per_batch, q_row0,
                                int(causal), k, thr.ctypes.data_as(f32p),
                                idx.ctypes.data_as(i32p), cnt.ctypes.data_as(i32p), idx_cap)
    if rc != 0:
        raise ValueError(f"oracle_topk_select rejected arguments (k={k}, N={N})")
    return thr, idx, cnt


def topk_threshold(scores, k: int) -> torch.Tensor:
    """[..., N] -> [..., 1] k-th largest, the topk_avx512.cpp:226-253 contract."""
    t = torch.as_tensor(scores)
    thr, _, _ = topk_select(t, k, idx_cap=0)
    return torch.from_numpy(thr).reshape(*t.shape[:-1], 1)


# --------------------------------------------------------------------------
# torch restatement of the reference's torch variant, row-chunked
# --------------------------------------------------------------------------

def _f32(x: torch.Tensor) -> torch.Tensor:
    return x.detach().to("cpu", torch.float32)


def indexer_scores(q, k, w, rows: slice | None = None, *, T_k: int | None = None) -> torch.Tensor:
    """Scores for query rows ``rows`` (default all) of q:[B,T,H,d], k:[B,T,d], w:[B,T,H].

    lightning_indexer.py:26-33: dots = einsum(bthd,bsd->bths); relu; (w*relu).sum(h);
    masked_fill(s > t, -inf).  Returns [B, len(rows), T_k] float32.
    """
    q, k, w = _f32(q), _f32(k), _f32(w)
    B, T, H, d = q.shape
    T_k = k.shape[1] if T_k is None else T_k
    rows = rows or slice(0, T)
    t0, t1 = rows.start or 0, rows.stop if rows.stop is not None else T
    dots = torch.einsum("bthd,bsd->bths", q[:, t0:t1], k[:, :T_k])
    scores = (w[:, t0:t1].unsqueeze(-1) * torch.relu(dots)).sum(dim=2)
    t_idx = torch.arange(t0, t1).unsqueeze(1)
    s_idx = torch.arange(T_k).unsqueeze(0)
    return scores.masked_fill(s_idx > t_idx, float("-inf"))


def project(h, W_Q, W_K, W_W, num_heads: int, head_dim: int):
    """lightning_indexer.py:36-42."""
    B, T, _ = h.shape
    q = (h @ W_Q).view(B, T, num_heads, head_dim)
    return q, h @ W_K, h @ W_W


def select_threshold(scores: torch.Tensor, top_k: int) -> torch.Tensor:
    """dsa_attention.py:41-44: k_eff = min(k, T); thr = topk(scores, k_eff).values[..., -1:]."""
    k_eff = min(top_k, scores.shape[-1])
    return scores.topk(k_eff, dim=-1).values[..., -1:]


def _attend(scores_rows, thr, Q, K, V, t0, t1, scale):
    """dsa_attention.py:46-51 for query rows [t0, t1): keep = scores >= thr & s <= t."""
    T_k = K.shape[1]
    causal = torch.arange(T_k).unsqueeze(0) <= torch.arange(t0, t1).unsqueeze(1)
    sel = (scores_rows >= thr) & causal                                   # [B,R,Tk]
    logits = torch.einsum("bthd,bshd->bths", Q[:, t0:t1], K) * scale      # [B,R,HQ,Tk]
    logits = logits.masked_fill(~sel.unsqueeze(2), float("-inf"))
    attn = torch.softmax(logits, dim=-1)
    return torch.einsum("bths,bshd->bthd", attn, V)


def dsa_attention(q_idx, k_idx, w_idx, Q, K, V, top_k: int, *, rows: slice | None = None,
                  chunk: int = 256, return_parts: bool = False):
    """dsa_attention.py:35-52 (``dsa_attention_torch``), over query-row chunks.

    Returns O [B, len(rows), HQ, DV] float32 (and, with return_parts, the
    scores and thresholds of those rows).
    """
    Q, K, V = _f32(Q), _f32(K), _f32(V)
    B, T, HQ, DQ = Q.shape
    scale = 1.0 / math.sqrt(DQ)
    rows = rows or slice(0, T)
    t0, t1 = rows.start or 0, rows.stop if rows.stop is not None else T
    outs, sc, th = [], [], []
    for c0 in range(t0, t1, chunk):
        c1 = min(c0 + chunk, t1)
        s = indexer_scores(q_idx, k_idx, w_idx, slice(c0, c1))
        thr = select_threshold(s, top_k)
        outs.append(_attend(s, thr, Q, K, V, c0, c1, scale))
        if return_parts:
            sc.append(s)
            th.append(thr)
    O = torch.cat(outs, dim=1)
    if return_parts:
        return O, torch.cat(sc, dim=1), torch.cat(th, dim=1)
    return O


def sparse_attention_with_threshold(scores, threshold, Q, K, V, *, rows: slice | None = None,
                                    chunk: int = 256):
    """dsa_attention.py:234-324: attention with a given [B,T,1] threshold."""
    Q, K, V = _f32(Q), _f32(K), _f32(V)
    scores, threshold = _f32(scores), _f32(threshold)
    B, T, HQ, DQ = Q.shape
    scale = 1.0 / math.sqrt(DQ)
    rows = rows or slice(0, T)
    t0, t1 = rows.start or 0, rows.stop if rows.stop is not None else T
    outs = []
    for c0 in range(t0, t1, chunk):
        c1 = min(c0 + chunk, t1)
        outs.append(_attend(scores[:, c0 - t0:c1 - t0], threshold[:, c0 - t0:c1 - t0],
                            Q, K, V, c0, c1, scale))
    return torch.cat(outs, dim=1)


def attention_from_lists(idx, cnt, Q, K, V, b: int, t: int) -> torch.Tensor:
    """Attention of query (b, t) over an explicit key list (dsa_attention.py:72-87,
    the naive variant's gather form).  Returns [HQ, DV] float32."""
    Q, K, V = _f32(Q), _f32(K), _f32(V)
    sel = torch.as_tensor(np.asarray(idx[: int(cnt)]), dtype=torch.long)
    scale = 1.0 / math.sqrt(Q.shape[-1])
    logits = torch.einsum("hd,khd->kh", Q[b, t], K[b, sel]) * scale
    attn = torch.softmax(logits, dim=0)
    return torch.einsum("kh,khd->hd", attn, V[b, sel])


def topk_mask(scores: torch.Tensor, k: int) -> torch.Tensor:
    """lightning_indexer.py:137-144."""
    k_eff = min(k, scores.shape[-1])
    _, idx = scores.topk(k_eff, dim=-1)
    mask = torch.zeros_like(scores, dtype=torch.bool)
    mask.scatter_(-1, idx, True)
    return mask


# --------------------------------------------------------------------------
# seeded synthetic inputs (CPU generator, so every machine sees the same bits)
# --------------------------------------------------------------------------

def make_inputs(B, T, HI, DI, HQ, DQ, DV, *, dtype=torch.float32, seed0: int = 0,
                scale: float = 1.0, w_scale: float | None = None):
    """q_idx, k_idx, w_idx, Q, K, V from CPU generators seeded seed0..seed0+5.

    q/k/v ~ N(0,1)*scale in ``dtype``; w ~ N(0,1)/sqrt(HI) in fp32 (or *w_scale).
    """
    def rnd(shape, s):
        g = torch.Generator().manual_seed(seed0 + s)
        return torch.randn(shape, generator=g, dtype=torch.float32)

    ws = (1.0 / math.sqrt(HI)) if w_scale is None else w_scale
    q_idx = (rnd((B, T, HI, DI), 0) * scale).to(dtype)
    k_idx = (rnd((B, T, DI), 1) * scale).to(dtype)
    w_idx = rnd((B, T, HI), 2) * ws
    Q = (rnd((B, T, HQ, DQ), 3) * scale).to(dtype)
    K = (rnd((B, T, HQ, DQ), 4) * scale).to(dtype)
    V = rnd((B, T, HQ, DV), 5).to(dtype)
    return q_idx, k_idx, w_idx, Q, K, V
