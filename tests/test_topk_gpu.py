"""GPU: radix-select top-K (stage 2) against the oracle — bit-exact thresholds
and kept-index sets on identical fp32 scores."""
import numpy as np
import pytest
import torch

from conftest import golden, t
import dsa_oracle as o

pytestmark = pytest.mark.gpu


def run(scores_cpu, k, *, causal=False, q_row0=0, idx_cap=None, cuda="cuda:0"):
    from topk import topk_select
    thr, idx, cnt = topk_select(scores_cpu.to(cuda), k, causal=causal, q_row0=q_row0, idx_cap=idx_cap)
    return thr.cpu().numpy(), idx.cpu().numpy(), cnt.cpu().numpy()


def assert_same(scores_cpu, k, **kw):
    x = scores_cpu.reshape(-1, scores_cpu.shape[-1]) if not kw.get("causal") else scores_cpu
    rpb = scores_cpu.shape[-2] if kw.get("causal") else None
    thr, idx, cnt = run(scores_cpu, k, **kw)
    cap = idx.shape[1]
    othr, oidx, ocnt = o.topk_select(scores_cpu, k, causal=kw.get("causal", False),
                                     rows_per_batch=rpb, q_row0=kw.get("q_row0", 0), idx_cap=cap)
    assert np.array_equal(thr, othr), "thresholds differ"        # by value: -0.0 == +0.0
    assert np.array_equal(cnt, ocnt), "kept counts differ"
    for r in range(len(cnt)):
        n = min(cnt[r], cap)
        assert np.array_equal(idx[r, :n], oidx[r, :n]), f"row {r} index list differs"
    return thr, idx, cnt


@pytest.mark.parametrize("name", ["topk_randn", "topk_ties"])
def test_threshold_matches_reference_golden(cuda, name):
    from topk import topk_threshold, topk_threshold_batch_merge
    d = golden(name)
    x = t(d["x"], cuda)
    for i, k in enumerate(d["ks"]):
        want = d["thr"][i]
        assert np.array_equal(topk_threshold(x, int(k))[..., 0].cpu().numpy(), want), f"k={k}"
        assert np.array_equal(topk_threshold_batch_merge(x, int(k))[..., 0].cpu().numpy(), want)
        assert_same(t(d["x"]), int(k))


@pytest.mark.parametrize("N,k", [(1, 1), (7, 3), (128, 1), (128, 128), (1000, 17), (2048, 128),
                                 (4097, 64), (5000, 5000), (16384, 512), (20000, 2048), (40000, 999)])
def test_random_rows_exact(cuda, N, k):
    g = torch.Generator().manual_seed(N * 7 + k)
    rows = max(2, min(64, 400000 // N))
    x = torch.randn(rows, N, generator=g)
    thr, _, cnt = assert_same(x, k)
    assert np.array_equal(thr, x.topk(k, dim=-1).values[:, -1].numpy())
    assert (cnt >= k).all()


def test_tie_heavy_and_special_values(cuda):
    g = torch.Generator().manual_seed(11)
    x = torch.round(torch.randn(32, 3000, generator=g) * 3) / 4         # few distinct values
    x[0] = 0.0
    x[1] = -0.0
    x[2, ::2] = -0.0                                                     # -0.0 mixed with +0.0
    x[3] = float("-inf")
    x[4, 100:] = float("-inf")
    x[5] = float("inf")
    x[6, :10] = float("inf")
    x[7] = torch.finfo(torch.float32).max
    x[8] = -torch.finfo(torch.float32).tiny                              # subnormal-adjacent
    x[9, ::3] = 1e-45                                                    # denormals
    for k in (1, 5, 64, 100, 101, 2999, 3000):
        assert_same(x, k)


def test_causal_rows_and_offsets(cuda):
    g = torch.Generator().manual_seed(5)
    s = torch.randn(3, 300, 1000, generator=g)            # values above the diagonal are junk
    for q_row0 in (0, 37, 700):
        for k in (1, 32, 64, 301):
            thr, idx, cnt = assert_same(s, k, causal=True, q_row0=q_row0)
            tt = q_row0 + np.arange(300)
            valid = np.minimum(tt + 1, 1000)
            short = np.tile(valid < k, 3)
            assert np.isneginf(thr[short]).all()
            assert (cnt[short] == np.tile(valid, 3)[short]).all()


def test_truncated_lists(cuda):
    x = torch.zeros(4, 512)
    x[:, 7] = 1.0
    thr, idx, cnt = assert_same(x, 8, idx_cap=32)           # 511 zeros tie with the 8th largest
    assert (cnt == 512).all() and (idx[:, :32] == np.arange(32)).all()


def test_c2_full_size_properties(cuda):
    """Config c2: 64 x 2048 x 2048 fp32 N(0,1) with s > t = -inf, k = 128.

    Full size on the GPU: thresholds equal torch.topk's bit-for-bit; counts
    and index lists satisfy the selection rule everywhere; sampled rows match
    the oracle exactly."""
    from topk import topk_select
    B, T, k = 64, 2048, 128
    g = torch.Generator(device=cuda).manual_seed(0)
    s = torch.randn(B, T, T, device=cuda, generator=g)
    s.masked_fill_(~torch.ones(T, T, device=cuda, dtype=torch.bool).tril(), float("-inf"))
    thr, idx, cnt = topk_select(s, k)
    ref = s.topk(k, dim=-1).values[..., -1].reshape(-1)
    assert torch.equal(thr, ref)
    kept = (s >= thr.view(B, T, 1))
    assert torch.equal(cnt, kept.sum(-1).reshape(-1).int())
    rows = torch.arange(B * T, device=cuda)
    sel = torch.arange(T, device=cuda).unsqueeze(0) < cnt.unsqueeze(1)
    vals = s.reshape(B * T, T).gather(1, idx.long().clamp(0, T - 1))
    assert bool((vals >= thr.unsqueeze(1))[sel].all())
    d = idx[:, 1:].long() - idx[:, :-1].long()
    assert bool((d > 0)[sel[:, 1:]].all()), "index lists must be strictly ascending"
    pick = torch.tensor([0, 1, 127, 128, 4095, 77777, B * T - 1])
    sc = s.reshape(B * T, T)[pick].cpu()
    othr, oidx, ocnt = o.topk_select(sc, k)
    assert np.array_equal(thr[pick].cpu().numpy(), othr)
    for j, r in enumerate(pick.tolist()):
        assert np.array_equal(idx[r, : ocnt[j]].cpu().numpy(), oidx[j, : ocnt[j]])


@pytest.mark.parametrize("N,k", [(2048, 128), (9000, 512), (20000, 2048)])
def test_long_row_kernel_exact(cuda, N, k, monkeypatch):
    """The kernel for rows longer than the shared-memory cache, forced on
    shorter rows, gives the same exact result."""
    monkeypatch.setenv("DSA_TOPK_LONG_PATH", "1")
    g = torch.Generator().manual_seed(N + k)
    x = torch.randn(6, N, generator=g)
    x[0, ::2] = 0.0
    assert_same(x, k)
    s = torch.randn(2, 50, N, generator=g)
    assert_same(s, k, causal=True, q_row0=N - 40)


@pytest.mark.parametrize("N,k", [(100, 7), (512, 32), (512, 512), (300, 128)])
def test_block_kernel_on_short_rows_exact(cuda, N, k, monkeypatch):
    """Rows <= 512 normally run one warp per row; the CTA-per-row kernel,
    forced on them, gives the same exact result."""
    monkeypatch.setenv("DSA_TOPK_NO_WARP", "1")
    g = torch.Generator().manual_seed(N * 3 + k)
    x = torch.randn(40, N, generator=g)
    x[3] = torch.round(x[3])
    assert_same(x, k)
    s = torch.randn(3, 64, N, generator=g)
    assert_same(s, min(k, N), causal=True, q_row0=max(0, N - 70))


@pytest.mark.parametrize("N,k", [(600, 32), (2048, 128), (4096, 512)])
def test_cta_kernel_on_mid_rows_exact(cuda, N, k, monkeypatch):
    """Rows of 513..4096 normally run one warp per row; the CTA-per-row
    kernel, forced on them, gives the same exact result."""
    monkeypatch.setenv("DSA_TOPK_NO_WL2", "1")
    g = torch.Generator().manual_seed(N + 5 * k)
    x = torch.randn(20, N, generator=g)
    x[2] = torch.round(x[2] * 2)
    assert_same(x, k)
    s = torch.randn(2, 30, N, generator=g)
    assert_same(s, k, causal=True, q_row0=N - 25)
