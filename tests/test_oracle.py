"""CPU: the oracle against the reference's own outputs (golden fixtures)."""
import glob
import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN, golden, t
import dsa_oracle as o


@pytest.mark.parametrize("name", ["topk_randn", "topk_ties"])
def test_topk_oracle_matches_reference_thresholds(name):
    d = golden(name)
    x = d["x"].reshape(-1, d["x"].shape[-1])
    for i, k in enumerate(d["ks"]):
        thr, idx, cnt = o.topk_select(x, int(k))
        assert np.array_equal(thr, d["thr"][i].reshape(-1)), f"k={k}"
        # kept set = {s: x[s] >= thr}, ascending
        for r in range(x.shape[0]):
            want = np.nonzero(x[r] >= thr[r])[0]
            assert cnt[r] == len(want) and np.array_equal(idx[r, : cnt[r]], want)
            assert cnt[r] >= k


def test_topk_oracle_causal_rows():
    g = torch.Generator().manual_seed(3)
    s = torch.randn(2, 40, 40, generator=g)
    full = s.masked_fill(torch.ones(40, 40).tril() == 0, float("-inf"))
    thr_c, idx_c, cnt_c = o.topk_select(s, 8, causal=True, rows_per_batch=40)   # junk above diag
    thr_f, idx_f, cnt_f = o.topk_select(full, 8)
    assert np.array_equal(thr_c, thr_f)
    tv = full.topk(8, dim=-1).values[..., -1].reshape(-1).numpy()
    assert np.array_equal(thr_c, tv)
    for r in range(80):
        tt = r % 40
        want = np.nonzero((full.reshape(80, 40)[r].numpy() >= thr_f[r]) & (np.arange(40) <= tt))[0]
        assert np.array_equal(idx_c[r, : cnt_c[r]], want)


@pytest.mark.parametrize("name", sorted(os.path.basename(p)[:-4] for p in glob.glob(os.path.join(GOLDEN, "indexer_*.npz"))))
def test_indexer_oracle_matches_reference(name):
    d = golden(name)
    out = o.indexer_scores(t(d["q"]), t(d["k"]), t(d["w"]))
    ref = t(d["scores"])
    fin = torch.isfinite(ref)
    assert torch.equal(fin, torch.isfinite(out))
    assert torch.allclose(out[fin], ref[fin], rtol=1e-5, atol=1e-5)
    assert torch.equal(o.topk_mask(out, 8), t(d["mask8"])) or \
        (o.topk_mask(out, 8) == t(d["mask8"])).float().mean() > 0.99


def test_project_oracle_matches_reference():
    d = golden("project")
    q, k, w = o.project(t(d["h"]), t(d["W_Q"]), t(d["W_K"]), t(d["W_W"]), int(d["H"]), int(d["d"]))
    out = o.indexer_scores(q, k, w)
    ref = t(d["scores"])
    fin = torch.isfinite(ref)
    assert (out[fin] - ref[fin]).abs().max() < 1e-4


@pytest.mark.parametrize("name", sorted(os.path.basename(p)[:-4] for p in glob.glob(os.path.join(GOLDEN, "dsa_*.npz"))))
def test_dsa_oracle_matches_reference(name):
    d = golden(name)
    args = [t(d[n]) for n in ("q_idx", "k_idx", "w_idx", "Q", "K", "V")]
    O, sc, thr = o.dsa_attention(*args, int(d["top_k"]), chunk=37, return_parts=True)
    assert (O - t(d["out"])).abs().max() < 1e-5
    assert torch.equal(thr, t(d["thr"]))
    if "out_naive" in d:
        assert (O - t(d["out_naive"])).abs().max() < 1e-4
    # threshold form and list form of the oracle agree with it
    O2 = o.sparse_attention_with_threshold(sc, thr, *args[3:])
    assert (O2 - O).abs().max() < 1e-5
    B, T = sc.shape[:2]
    th, idx, cnt = o.topk_select(sc, min(int(d["top_k"]), T), causal=True, rows_per_batch=T)
    assert np.array_equal(th, thr.reshape(-1).numpy())
    for r in range(0, B * T, max(1, B * T // 23)):
        b, tt = divmod(r, T)
        Or = o.attention_from_lists(idx[r], cnt[r], *args[3:], b, tt)
        assert (Or - O[b, tt]).abs().max() < 1e-5
