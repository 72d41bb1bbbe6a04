"""GPU: edge semantics of the selection and of the entry points.

NaN scores follow the reference's torch variant (dsa_attention.py:41-46):
torch.topk ranks every NaN above +inf, so NaNs push the k-th largest up, and
the kept set is `scores >= threshold`, which is false for NaN: a NaN is never
kept, and a NaN threshold (k or more NaNs in a row) keeps nothing.  Every
top-K kernel (chosen by row length) is checked bit for bit against the C
oracle and torch.topk on rows holding +NaN, -NaN and NaN payloads.

Empty calls (B = 0 or T_q = 0) are no-ops that return DSA_OK without a
workspace, like dsa_indexer_scores."""
import ctypes
import os

import numpy as np
import pytest
import torch

import dsa_oracle as o

pytestmark = pytest.mark.gpu


def _nan_rows(rows, N, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(rows, N, generator=g)
    x[0, :: max(1, N // 7)] = float("nan")                      # a few NaNs
    x[1, : N // 2] = float("nan")                                # NaNs fill the top ranks
    x[2] = float("nan")                                          # all NaN: threshold NaN
    x[3, 1::5] = -float("nan")                                   # -NaN (sign bit set)
    bits = x[4].view(torch.int32)
    bits[:: max(1, N // 3)] = 0x7fc12345                        # NaN payloads
    x[5, ::4] = float("inf")
    x[5, 2::4] = float("nan")                                    # +inf beside NaN
    x[6, 3] = float("nan")
    return x


def _same_nan_aware(a, b):
    return np.array_equal(np.asarray(a), np.asarray(b), equal_nan=True)


@pytest.mark.parametrize("N,k", [(100, 7), (300, 64), (2000, 128), (6000, 512), (20000, 2048),
                                 (40000, 999)])
def test_nan_rows_match_oracle_and_torch(cuda, N, k):
    from topk import topk_select
    x = _nan_rows(8, N, seed=N + k)
    thr, idx, cnt = topk_select(x.to(cuda), k)
    othr, oidx, ocnt = o.topk_select(x, k, idx_cap=N)
    assert _same_nan_aware(thr.cpu().numpy(), othr)
    assert _same_nan_aware(thr.cpu().numpy(), x.topk(k, dim=-1).values[:, -1].numpy())
    assert np.array_equal(cnt.cpu().numpy(), ocnt)
    want = (x >= torch.from_numpy(othr).unsqueeze(1)).sum(1).numpy()   # NaN >= anything is False
    assert np.array_equal(ocnt, want)
    for r in range(x.shape[0]):
        n = int(ocnt[r])
        assert np.array_equal(idx[r, :n].cpu().numpy(), oidx[r, :n]), f"row {r}"
    assert ocnt[2] == 0 and np.isnan(othr[2])


@pytest.mark.parametrize("T,k,q_row0", [(300, 32, 0), (2000, 128, 100), (6000, 512, 0), (20000, 2048, 19900)])
def test_nan_rows_bitmap_and_causal(cuda, T, k, q_row0):
    """Causal rows with NaNs: the bitmap form (the path the tensor-core
    attention reads) holds exactly the kept set."""
    import _native
    from topk import topk_select_bitmap
    rows = 8
    x = _nan_rows(rows, T, seed=T + 1).view(1, rows, T)
    thr, cnt, bits = topk_select_bitmap(x.to(cuda), k, q_row0=q_row0)
    othr, _, ocnt = o.topk_select(x, k, causal=True, rows_per_batch=rows, q_row0=q_row0, idx_cap=1)
    assert _same_nan_aware(thr.cpu().numpy(), othr)
    assert np.array_equal(cnt.cpu().numpy(), ocnt)
    t = q_row0 + torch.arange(rows).view(rows, 1)
    keep = (torch.arange(T).view(1, T) <= t) & (x[0] >= torch.from_numpy(othr).view(rows, 1))
    words = _native.bitmap_words(T)
    pad = np.zeros((rows, words * 32), dtype=np.uint64)
    pad[:, :T] = keep.numpy()
    want = (pad.reshape(rows, words, 32) << np.arange(32, dtype=np.uint64)).sum(-1).astype(np.uint32)
    assert np.array_equal(bits.cpu().numpy().view(np.uint32), want)


def test_forward_nan_threshold_row_gives_nan_like_reference(cuda):
    """A row whose k largest scores are all NaN keeps nothing; the reference's
    softmax over all -inf logits returns NaN there, and so does stage 3."""
    from dsa_attention import sparse_attention_with_threshold_triton
    B, T, H, D = 1, 256, 2, 64
    _, _, _, Q, K, V = o.make_inputs(B, T, 1, 8, H, D, D, dtype=torch.bfloat16)
    sc = torch.randn(B, T, T, generator=torch.Generator().manual_seed(3))
    sc = sc.masked_fill(~torch.ones(T, T, dtype=torch.bool).tril(), float("-inf"))
    sc[0, 200, :150] = float("nan")
    thr = o.select_threshold(sc, 16)
    assert torch.isnan(thr[0, 200]).all()
    ref = o.sparse_attention_with_threshold(sc, thr, Q, K, V)
    for gather in ("0", "1"):
        os.environ["DSA_ATTN_GATHER"] = gather
        try:
            out = sparse_attention_with_threshold_triton(sc.to(cuda), thr.to(cuda), Q.to(cuda), K.to(cuda),
                                                         V.to(cuda)).cpu()
        finally:
            os.environ.pop("DSA_ATTN_GATHER")
        assert torch.isnan(out[0, 200]).all() and torch.isnan(ref[0, 200]).all()
        fin = torch.ones(T, dtype=torch.bool)
        fin[200] = False
        assert ((out[0, fin] - ref[0, fin]).abs() <= 1e-3 + 2e-2 * ref[0, fin].abs()).all()


@pytest.mark.parametrize("B,T_q", [(0, 64), (2, 0)])
def test_empty_calls_return_ok_without_workspace(cuda, B, T_q):
    import _native
    L = _native.lib()
    T_k, HI, DI, HQ, D, k = 64, 2, 32, 2, 32, 8
    q = torch.zeros(max(B, 1), max(T_q, 1), HI, DI, device=cuda)
    kk = torch.zeros(max(B, 1), T_k, DI, device=cuda)
    w = torch.zeros(max(B, 1), max(T_q, 1), HI, device=cuda)
    Q = torch.zeros(max(B, 1), max(T_q, 1), HQ, D, device=cuda)
    K = torch.zeros(max(B, 1), T_k, HQ, D, device=cuda)
    O = torch.zeros(max(B, 1), max(T_q, 1), HQ, D, device=cuda)
    p = lambda x: ctypes.c_void_p(x.data_ptr())
    s = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = L.dsa_forward(p(q), p(kk), p(w), p(Q), p(K), p(K), p(O), B, T_q, T_k, 0, HI, DI, HQ, D, D, k,
                       _native.DSA_F32, _native.DSA_F32, None, 0, s)
    assert rc == _native.DSA_OK, L.dsa_last_error_string()
    rc = L.dsa_forward_noalloc(p(q), p(kk), p(w), p(Q), p(K), p(K), p(O), B, T_q, T_k, 0, HI, DI, HQ, D,
                               D, k, _native.DSA_F32, _native.DSA_F32, s)
    assert rc == _native.DSA_OK, L.dsa_last_error_string()
    # the Python entry point too (its workspace for an empty call is empty)
    from dsa_attention import dsa_forward
    out = dsa_forward(q[:B, :T_q], kk[:B], w[:B, :T_q], Q[:B, :T_q], K[:B], K[:B], k)
    assert out.shape == (B, T_q, HQ, D)
