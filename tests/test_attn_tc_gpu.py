"""GPU: the tensor-core attention stage (kept-set bitmap + tcgen05 masked
flash attention) against the oracle.

The bitmap is integer work and must match bit for bit.  The attention rounds
its softmax weights to the input dtype before the P.V product, so it is held
to the north-star bf16/fp16 tolerance elementwise (|err| <= 1e-3 + 2e-2 |ref|),
and it is also compared with the fp32 gather kernel on identical kept sets."""
import math

import numpy as np
import pytest
import torch

import dsa_oracle as o
from conftest import assert_close_elementwise

pytestmark = pytest.mark.gpu


def _bits_ref(sc: torch.Tensor, thr: torch.Tensor, q_row0: int, words: int) -> np.ndarray:
    """Bitmap of (s <= q_row0 + i) & (scores >= thr), built with numpy."""
    B, T_q, T_k = sc.shape
    t = q_row0 + torch.arange(T_q).view(1, T_q, 1)
    s = torch.arange(T_k).view(1, 1, T_k)
    keep = ((s <= t) & (sc >= thr.view(B, T_q, 1))).reshape(B * T_q, T_k).numpy()
    pad = np.zeros((B * T_q, words * 32), dtype=np.uint64)
    pad[:, :T_k] = keep
    w = (pad.reshape(B * T_q, words, 32) << np.arange(32, dtype=np.uint64)).sum(-1)
    return w.astype(np.uint32).view(np.int32)


def _case(B, T_q, T_k, HQ, D, k, dtype, q_row0, seed):
    g = torch.Generator().manual_seed(seed)
    sc = torch.randn(B, T_q, T_k, generator=g)
    # ties: quantise a third of the rows so equal scores straddle the threshold
    sc[:, ::3] = (sc[:, ::3] * 4).round() / 4
    t = q_row0 + torch.arange(T_q).view(1, T_q, 1)
    causal = torch.arange(T_k).view(1, 1, T_k) <= t
    masked = torch.where(causal, sc, torch.full_like(sc, -math.inf))
    kk = min(k, T_k)
    thr = masked.topk(kk, dim=-1).values[..., -1]
    # rows with fewer than k causal keys keep all of them
    thr = torch.where(torch.isfinite(thr), thr, torch.full_like(thr, -math.inf))
    Q = torch.randn(B, T_q, HQ, D, generator=g).to(dtype)
    K = torch.randn(B, T_k, HQ, D, generator=g).to(dtype)
    V = torch.randn(B, T_k, HQ, D, generator=g).to(dtype)
    return sc, thr, Q, K, V


def _oracle(sc, thr, Q, K, V, q_row0):
    """fp32 attention over the kept set of each row (the oracle's _attend rule)."""
    B, T_q, T_k = sc.shape
    D = Q.shape[-1]
    t = q_row0 + torch.arange(T_q).view(1, T_q, 1)
    keep = (torch.arange(T_k).view(1, 1, T_k) <= t) & (sc >= thr.view(B, T_q, 1))
    logits = torch.einsum("bthd,bshd->bhts", Q.float(), K.float()) / math.sqrt(D)
    logits = logits.masked_fill(~keep.unsqueeze(1), -math.inf)
    p = torch.softmax(logits, dim=-1)
    return torch.einsum("bhts,bshd->bthd", p, V.float())


CASES = [
    # B, T_q, T_k, HQ, D, k, dtype, q_row0
    (1, 256, 256, 2, 128, 32, torch.bfloat16, 0),
    (2, 300, 300, 3, 64, 40, torch.bfloat16, 0),      # ragged tiles, D=64
    (1, 200, 777, 2, 128, 64, torch.float16, 577),    # a row block at an offset, T_k ragged
    (1, 1024, 1024, 4, 128, 96, torch.bfloat16, 0),
    (2, 513, 513, 2, 64, 513, torch.float16, 0),      # k >= T: dense causal attention
    (1, 64, 4000, 1, 128, 300, torch.bfloat16, 3936), # one short query tile, many key blocks
]


@pytest.mark.parametrize("B,T_q,T_k,HQ,D,k,dtype,q_row0", CASES)
def test_bitmap_and_tc_attention_match_oracle(cuda, B, T_q, T_k, HQ, D, k, dtype, q_row0):
    import _native
    from dsa_attention import kept_bitmap, sparse_attention_with_bitmap
    sc, thr, Q, K, V = _case(B, T_q, T_k, HQ, D, k, dtype, q_row0, seed=T_q + T_k + D)
    bits = kept_bitmap(sc.to(cuda), thr.to(cuda), q_row0=q_row0)
    words = _native.bitmap_words(T_k)
    assert bits.shape == (B * T_q, words) and words % 4 == 0
    assert np.array_equal(bits.cpu().numpy(), _bits_ref(sc, thr, q_row0, words))
    out = sparse_attention_with_bitmap(bits, Q.to(cuda), K.to(cuda), V.to(cuda), q_row0=q_row0).cpu()
    ref = _oracle(sc, thr, Q, K, V, q_row0)
    assert torch.isfinite(out).all()
    assert_close_elementwise(out, ref, what="tensor-core attention vs oracle")


def test_tc_attention_agrees_with_gather_kernel(cuda, monkeypatch):
    """Same kept sets through both stage-3 kernels (bitmap/tensor cores vs threshold/gather)."""
    from dsa_attention import sparse_attention_with_threshold_triton
    sc, thr, Q, K, V = _case(2, 640, 640, 4, 128, 64, torch.bfloat16, 0, seed=11)
    args = (sc.to(cuda), thr.to(cuda), Q.to(cuda), K.to(cuda), V.to(cuda))
    tc = sparse_attention_with_threshold_triton(*args)
    monkeypatch.setenv("DSA_ATTN_GATHER", "1")
    ga = sparse_attention_with_threshold_triton(*args)
    assert_close_elementwise(tc, ga, what="tensor-core vs gather attention")


@pytest.mark.parametrize("B,T,HI,DI,HQ,D,k,dtype", [
    (1, 1024, 8, 128, 4, 128, 64, torch.bfloat16),
    (2, 700, 4, 64, 2, 64, 50, torch.float16),
])
def test_forward_tc_path_matches_oracle_and_gather(cuda, B, T, HI, DI, HQ, D, k, dtype, monkeypatch):
    from dsa_attention import dsa_forward
    args = [x.to(cuda) for x in o.make_inputs(B, T, HI, DI, HQ, D, D, dtype=dtype, seed0=5)]
    out = dsa_forward(*args, k)
    monkeypatch.setenv("DSA_ATTN_GATHER", "1")
    ga = dsa_forward(*args, k)
    assert_close_elementwise(out, ga, what="forward: tensor-core vs gather stage 3")
    # the oracle's attention on the GPU's own scores and thresholds (the bf16
    # indexer's sums round differently from the fp32 oracle's, which can move
    # a key across a near-tied threshold)
    from lightning_indexer import indexer_scores
    from topk import topk_select
    sc = indexer_scores(*args[:3])
    thr, _, _ = topk_select(sc, k, causal=True, return_idx=False)
    ref = o.sparse_attention_with_threshold(sc.cpu(), thr.cpu().view(B, T, 1), *(a.cpu() for a in args[3:]))
    assert_close_elementwise(out, ref, what="forward vs oracle on the GPU's scores")


def test_bitmap_entry_points_reject_bad_arguments(cuda):
    import _native
    from dsa_attention import sparse_attention_with_bitmap
    Q = torch.zeros(1, 128, 1, 32, device=cuda, dtype=torch.bfloat16)   # D=32: not on the tensor cores
    bits = torch.zeros(128, _native.bitmap_words(128), device=cuda, dtype=torch.int32)
    with pytest.raises(RuntimeError, match="bf16/fp16"):
        sparse_attention_with_bitmap(bits, Q, Q, Q)
    sc = torch.zeros(1, 128, 128, device=cuda)
    thr = torch.zeros(128, device=cuda)
    short = torch.zeros(128, 2, device=cuda, dtype=torch.int32)          # fewer words than needed
    with pytest.raises(AssertionError, match="words_per_row"):
        _native.kept_bitmap(sc, thr, short)


def test_attention_wait_timeout_is_reported_and_recoverable(cuda, monkeypatch):
    """Test hook DSA_TEST_ATTN_STALL: the producer issues no loads, every wait
    runs out after 20 ms, the kernel returns and the status reports it."""
    import _native
    from dsa_attention import kept_bitmap, sparse_attention_with_bitmap
    sc, thr, Q, K, V = _case(1, 256, 256, 2, 64, 32, torch.bfloat16, 0, seed=3)
    bits = kept_bitmap(sc.to(cuda), thr.to(cuda))
    Q, K, V = Q.to(cuda), K.to(cuda), V.to(cuda)
    assert _native.device_status() == _native.DSA_OK
    monkeypatch.setenv("DSA_TEST_ATTN_STALL", "1")
    sparse_attention_with_bitmap(bits, Q, K, V)
    assert _native.device_status() == _native.DSA_ERR_TIMEOUT
    assert _native.device_status() == _native.DSA_OK
    monkeypatch.delenv("DSA_TEST_ATTN_STALL")
    out = sparse_attention_with_bitmap(bits, Q, K, V).cpu()
    assert _native.device_status() == _native.DSA_OK
    ref = _oracle(sc, thr, Q.cpu(), K.cpu(), V.cpu(), 0)
    assert_close_elementwise(out, ref, what="attention after a timeout")


@pytest.mark.parametrize("B,T_q,T_k,k,q_row0,causal", [
    (1, 64, 6000, 700, 5936, True),     # 4K-32K rows: the bitmap comes from the top-K kernel
    (2, 40, 9000, 64, 8960, True),
    (1, 300, 300, 20, 0, True),         # short rows: top-K kernel, then the bitmap kernel
    (3, 5, 5000, 100, 0, False),        # full rows, no causal limit
    (1, 48, 7000, 3000, 6952, True),    # a third of the scores -inf: thresholds fall in the -inf bin
])
def test_topk_bitmap_equals_threshold_then_bitmap(cuda, B, T_q, T_k, k, q_row0, causal):
    from dsa_attention import kept_bitmap
    from topk import topk_select, topk_select_bitmap
    g = torch.Generator(device=cuda).manual_seed(T_k)
    sc = torch.randn(B, T_q, T_k, generator=g, device=cuda)
    sc[:, ::2] = (sc[:, ::2] * 8).round() / 8            # ties at the threshold
    if k >= 3000:
        sc[..., ::3] = -math.inf
    thr, cnt, bits = topk_select_bitmap(sc, k, causal=causal, q_row0=q_row0)
    thr2, _, cnt2 = topk_select(sc, k, causal=causal, q_row0=q_row0, idx_cap=32)
    assert torch.equal(thr, thr2) and torch.equal(cnt, cnt2)
    if causal:
        ref = kept_bitmap(sc, thr, q_row0=q_row0)
    else:
        ref = torch.from_numpy(_bits_ref(sc.cpu(), thr.cpu(), T_k, bits.shape[1])).to(cuda)
    assert torch.equal(bits, ref)


@pytest.mark.parametrize("k", [5, 700, 2000, 4999])
def test_topk_bitmap_special_values(cuda, k):
    """+inf, -inf and both signs of zero at the threshold (+0 and -0 tie),
    on 5000-entry rows, which take the one-sweep bitmap path of the top-K
    kernel; the result must equal the list-mode selection."""
    from dsa_attention import kept_bitmap
    from topk import topk_select, topk_select_bitmap
    g = torch.Generator(device=cuda).manual_seed(k)
    sc = torch.randn(2, 3, 5000, generator=g, device=cuda).round()   # many exact ties, zeros of both signs
    sc[0, 0, ::7] = math.inf
    sc[0, 1, ::3] = -math.inf
    sc[1, :, ::2] = -0.0
    sc[1, 2] = 0.0
    sc[1, 2, ::5] = -0.0
    thr, cnt, bits = topk_select_bitmap(sc, k, causal=False)
    thr2, _, cnt2 = topk_select(sc, k, causal=False, idx_cap=32)
    assert torch.equal(thr, thr2) and torch.equal(cnt, cnt2)
    ref = torch.from_numpy(_bits_ref(sc.cpu(), thr.cpu(), 5000, bits.shape[1])).to(cuda)
    assert torch.equal(bits, ref)
    pop = sum(((bits >> b) & 1).sum(1) for b in range(32))
    assert torch.equal(pop, cnt.long())


@pytest.mark.parametrize("k", [1, 700, 2048, 9999])
def test_topk_bitmap_bin_edges_long_rows(cuda, k):
    """20,000-entry rows (the kernel variant c5 uses) whose values sit on the
    edges of the first-digit bins (1.0, 1.25, -0.75, ... have two mantissa
    bits), with both zeros and denormals: the float-compare sweep must keep
    exactly the keys a key compare keeps, with the threshold of torch.topk."""
    from topk import topk_select, topk_select_bitmap
    g = torch.Generator(device=cuda).manual_seed(k)
    edges = torch.tensor([0.5, 0.75, 1.0, 1.25, 1.5, 1.75, 2.0, -0.5, -0.75, -1.0, 0.0, -0.0,
                          1e-40, -1e-40, 3.0, 2.5], device=cuda)
    n = 20000
    pick = torch.randint(0, len(edges), (2, 8, n), generator=g, device=cuda)
    sc = edges[pick]
    noisy = torch.rand(2, 8, n, generator=g, device=cuda) < 0.3
    sc = torch.where(noisy, torch.randn(2, 8, n, generator=g, device=cuda), sc)
    sc[1, 3] = torch.randn(n, generator=g, device=cuda) * 1e-39      # denormal row
    thr, cnt, bits = topk_select_bitmap(sc, k, causal=False)
    thr2, _, cnt2 = topk_select(sc, k, causal=False, idx_cap=32)
    assert torch.equal(thr, thr2) and torch.equal(cnt, cnt2)
    kth = sc.topk(k, dim=-1).values[..., -1:]
    assert torch.equal(thr.view_as(kth), kth)
    ref = torch.from_numpy(_bits_ref(sc.cpu(), thr.cpu(), n, bits.shape[1])).to(cuda)
    assert torch.equal(bits, ref)


@pytest.mark.parametrize("levels", [3, 40])
def test_topk_bitmap_threshold_bin_overflow(cuda, levels):
    """Rows of 4K-8K entries whose threshold bin holds more keys than the
    candidate buffer (scores drawn from a few values): the kernel takes its
    exact path without candidates and must still write the same bitmap."""
    from topk import topk_select, topk_select_bitmap
    g = torch.Generator(device=cuda).manual_seed(levels)
    sc = torch.randint(0, levels, (2, 64, 7000), generator=g, device=cuda).float() / levels
    thr, cnt, bits = topk_select_bitmap(sc, 900, causal=True, q_row0=6936)
    thr2, _, cnt2 = topk_select(sc, 900, causal=True, q_row0=6936, idx_cap=32)
    assert torch.equal(thr, thr2) and torch.equal(cnt, cnt2)
    ref = torch.from_numpy(_bits_ref(sc.cpu(), thr.cpu(), 6936, bits.shape[1])).to(cuda)
    assert torch.equal(bits, ref)


def test_row_blocks_of_the_tc_forward_equal_the_whole(cuda):
    """q_row0 offsets on the tensor-core path: query row blocks that do not
    start on a tile boundary give the rows of the whole forward bit for bit
    (each row's softmax does not depend on how rows are grouped into tiles)."""
    from dsa_attention import dsa_forward
    qi, ki, wi, Q, K, V = (x.to(cuda) for x in o.make_inputs(1, 900, 4, 128, 2, 128, 128,
                                                            dtype=torch.bfloat16, seed0=21))
    whole = dsa_forward(qi, ki, wi, Q, K, V, 100)
    parts = [dsa_forward(qi[:, a:b].contiguous(), ki, wi[:, a:b].contiguous(), Q[:, a:b].contiguous(), K, V,
                         100, q_row0=a)
             for a, b in [(0, 77), (77, 400), (400, 900)]]
    assert torch.equal(torch.cat(parts, 1), whole)


@pytest.mark.parametrize("T,window,stride", [(2048, 200, 512), (1500, 64, 300)])
def test_block_skipping_is_exact_on_structured_selections(cuda, T, window, stride, monkeypatch):
    """Kept sets of a local window plus strided key blocks (most 128x128 tiles
    hold no kept key): the attention that skips empty key blocks equals the one
    that processes every causal block bit for bit, and the oracle elementwise."""
    from dsa_attention import kept_bitmap, sparse_attention_with_bitmap
    B, HQ, D, k = 1, 2, 128, 256
    t = torch.arange(T).view(T, 1)
    s = torch.arange(T).view(1, T)
    g = torch.Generator().manual_seed(T)
    sc = torch.randn(1, T, T, generator=g) * 0.1
    sc += ((t - s >= 0) & (t - s < window)).float() * 10 + ((s % stride) < 64).float() * 5
    thr = sc.masked_fill(s > t, float("-inf")).topk(k, dim=-1).values[..., -1]
    thr = torch.where(torch.isfinite(thr), thr, torch.full_like(thr, float("-inf")))
    Q, K, V = (torch.randn(B, T, HQ, D, generator=g).to(torch.bfloat16) for _ in range(3))
    bits = kept_bitmap(sc.to(cuda), thr.to(cuda))
    args = (bits, Q.to(cuda), K.to(cuda), V.to(cuda))
    skipped = sparse_attention_with_bitmap(*args)
    monkeypatch.setenv("DSA_ATTN_NO_SKIP", "1")
    full = sparse_attention_with_bitmap(*args)
    assert torch.equal(skipped, full)
    assert_close_elementwise(skipped, _oracle(sc, thr, Q, K, V, 0), what="structured selection vs oracle")
