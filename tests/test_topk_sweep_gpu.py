"""GPU: the two-kernel bitmap top-K (sweep + per-row resolver, taken when a
workspace is given) equals the one-kernel form bit for bit -- thresholds,
counts and every bitmap word -- on rows of 4K-32K entries, and its thresholds
equal torch.topk's.  Data: Gaussian rows, rows with many exact (and signed)
zeros, tie-heavy rows, heavy-tailed rows whose threshold bin overflows the
candidate list, rows holding NaN and infinities, and row blocks."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def make(kind, B, Tq, T, seed, cuda):
    g = torch.Generator(device=cuda).manual_seed(seed)
    x = torch.randn((B, Tq, T), generator=g, device=cuda)
    if kind == "relu":            # half exact zeros, some of them -0.0
        x = x.clamp_min(0) * torch.where(torch.rand(x.shape, generator=g, device=cuda) < 0.5, -1.0, 1.0)
    elif kind == "ties":
        x = (x * 4).round() / 4
    elif kind == "heavy":         # wide dynamic range: crowded first-digit bins
        x = torch.exp(x * 6)
    elif kind == "wide":          # like the indexer's c5 scores: the threshold's bin holds ~3% of a row
        x = 6.0 + 8.0 * x
    elif kind == "special":
        x[:, ::97, ::13] = float("nan")
        x[:, 5::89, 3::17] = float("inf")
        x[:, 7::83, 1::19] = float("-inf")
        x[:, 11::71, :] = 0.0
    return x


def both(x, k, q_row0):
    from topk import topk_select_bitmap
    a = topk_select_bitmap(x, k, q_row0=q_row0, workspace=True)
    b = topk_select_bitmap(x, k, q_row0=q_row0, workspace=False)
    return a, b


@pytest.mark.parametrize("kind", ["randn", "relu", "ties", "heavy", "wide", "special"])
@pytest.mark.parametrize("B,Tq,T,k,q_row0", [(1, 8192, 8192, 512, 0), (2, 3000, 6000, 300, 3000),
                                              (1, 2048, 32768, 2048, 30720), (1, 1024, 16384, 4096, 9000)])
def test_sweep_resolve_equals_one_kernel(cuda, kind, B, Tq, T, k, q_row0):
    x = make(kind, B, Tq, T, B * 131 + Tq + k, cuda)
    (t1, c1, b1), (t2, c2, b2) = both(x, k, q_row0)
    assert torch.equal(t1.view(torch.int32), t2.view(torch.int32)), "thresholds differ"
    assert torch.equal(c1, c2), "counts differ"
    assert torch.equal(b1, b2), "bitmaps differ"
    # thresholds against torch.topk on a few rows (causal entries only)
    for r in (0, Tq // 3, Tq - 1):
        t = q_row0 + r
        row = x[0, r, : t + 1]
        if t + 1 < k:
            continue
        want = row.topk(k).values[-1]
        got = t1[r]
        assert (torch.isnan(want) and torch.isnan(got)) or bool(want == got), (r, want.item(), got.item())


def test_sweep_resolve_row_blocks(cuda):
    """Two row blocks of one sequence as one call (row_bstep) equal two calls."""
    import _native
    T, Tq, k = 16384, 1024, 1024
    g = torch.Generator(device=cuda).manual_seed(5)
    x = torch.randn((2, Tq, T), generator=g, device=cuda)
    q0, step = 2048, 9000
    words = _native.bitmap_words(T)
    ws = torch.empty(_native.topk_select_bitmap_workspace_bytes(2 * Tq, words), device=cuda, dtype=torch.uint8)
    thr = torch.empty(2 * Tq, device=cuda)
    cnt = torch.empty(2 * Tq, device=cuda, dtype=torch.int32)
    bits = torch.empty((2 * Tq, words), device=cuda, dtype=torch.int32)
    _native.topk_select_bitmap(x, k, thr, bits, cnt, q_row0=q0, row_bstep=step, workspace=ws)
    from topk import topk_select_bitmap
    for i, a in enumerate((q0, q0 + step)):
        t1, c1, b1 = topk_select_bitmap(x[i:i + 1], k, q_row0=a, workspace=False)
        sl = slice(i * Tq, (i + 1) * Tq)
        assert torch.equal(thr[sl].view(torch.int32), t1.view(torch.int32)) and torch.equal(cnt[sl], c1) and torch.equal(bits[sl], b1), i
