"""GPU: the forward at BASELINE.json's full sizes (configs c4 and c5).

A CPU oracle cannot run these sizes whole, so every row is checked through
size-independent properties of the GPU's own stage outputs, and sampled rows
are checked against the oracle:
  - top-K on every row: the count of scores strictly above the threshold is
    < k, the count at or above it is >= min(k, t+1); the kept list is
    ascending, in 0..t, and holds exactly the positions >= threshold;
  - the kept-set bitmap of every row holds exactly cnt bits;
  - 64 sampled rows stratified over every batch: threshold and kept list
    bit-exact against the C oracle on the GPU's score row; indexer scores
    within the bf16 tolerance of the fp32 oracle; attention output within
    1e-3 + 2e-2 |O| elementwise of the oracle run on the GPU's kept set;
    and the pipeline's output equals the stage-by-stage one.
"""
import math

import numpy as np
import pytest
import torch

import dsa_oracle as o
from conftest import ATOL_16, assert_close_elementwise

pytestmark = pytest.mark.gpu

CONFIGS = {
    "c4": dict(B=4, T=8192, HI=16, DI=64, HQ=16, D=64, k=512),
    "c5": dict(B=1, T=32768, HI=64, DI=128, HQ=16, D=128, k=2048),
}


def _inputs(cfg, dev):
    g = torch.Generator(device=dev).manual_seed(7)
    B, T, HI, DI, HQ, D = (cfg[x] for x in ("B", "T", "HI", "DI", "HQ", "D"))
    rnd = lambda shape, sc=1.0, dt=torch.bfloat16: (torch.randn(shape, generator=g, device=dev) * sc).to(dt)
    return (rnd((B, T, HI, DI)), rnd((B, T, DI)), rnd((B, T, HI), 1 / math.sqrt(HI), torch.float32),
            rnd((B, T, HQ, D)), rnd((B, T, HQ, D)), rnd((B, T, HQ, D)))


@pytest.mark.parametrize("name", ["c4", "c5"])
def test_forward_full_size(cuda, name):
    import _native
    from dsa_attention import dsa_forward, kept_bitmap, sparse_attention_with_bitmap, sparse_attention_with_lists
    from lightning_indexer import indexer_scores
    from topk import idx_cap_for, topk_select
    cfg = CONFIGS[name]
    B, T, k = cfg["B"], cfg["T"], cfg["k"]
    args = _inputs(cfg, cuda)
    O = dsa_forward(*args, k)

    # stage by stage, keeping the intermediates
    sc = indexer_scores(*args[:3], fill_upper=False)
    cap = idx_cap_for(k, T)
    thr, idx, cnt = topk_select(sc, k, causal=True, idx_cap=cap)
    if _native.attn_tc_supported(args[3], args[5]):
        # bf16 heads of 64/128: dsa_forward's stage 3 is the tensor-core kernel over the bitmap
        O2 = sparse_attention_with_bitmap(kept_bitmap(sc, thr), *args[3:])
    else:
        O2 = sparse_attention_with_lists(idx, cnt, cap, sc, thr, *args[3:])
    assert torch.equal(O, O2), "dsa_forward differs from its own stages"
    assert torch.isfinite(O).all()

    # ---- size-independent top-K properties on every row
    rows = B * T
    t = torch.arange(T, device=cuda).repeat(B)
    s_pos = torch.arange(T, device=cuda)
    above = torch.zeros(rows, device=cuda, dtype=torch.int64)
    atleast = torch.zeros(rows, device=cuda, dtype=torch.int64)
    for r0 in range(0, rows, 1024):                    # chunks keep the masks small
        r1 = min(r0 + 1024, rows)
        blk = sc.view(rows, T)[r0:r1]
        causal = s_pos.unsqueeze(0) <= t[r0:r1].unsqueeze(1)
        th = thr[r0:r1].unsqueeze(1)
        above[r0:r1] = ((blk > th) & causal).sum(1)
        atleast[r0:r1] = ((blk >= th) & causal).sum(1)
    assert bool((above < k).all())
    assert bool((atleast >= torch.clamp(t + 1, max=k)).all())
    assert torch.equal(atleast, cnt.long())
    bits = kept_bitmap(sc, thr)
    pop = torch.zeros(rows, device=cuda, dtype=torch.int64)
    for sh in range(32):                                 # popcount, one bit position at a time
        pop += ((bits >> sh) & 1).sum(1)
    assert torch.equal(pop, cnt.long())
    n = torch.clamp(cnt.long(), max=cap)
    valid = torch.arange(cap, device=cuda).unsqueeze(0) < n.unsqueeze(1)
    il = idx.long()
    assert bool(((il <= t.unsqueeze(1)) | ~valid).all()) and bool(((il >= 0) | ~valid).all())
    asc = il[:, 1:] > il[:, :-1]
    assert bool((asc | ~valid[:, 1:]).all())

    # ---- sampled rows against the oracle: 64 rows stratified over every batch
    # (the edges of the causal ramp and evenly spaced positions between them)
    per_b = max(16, 64 // B)
    edges = [0, 1, k - 2, k - 1, k, T - 2, T - 1]
    spread = np.linspace(2, T - 3, per_b - len(edges)).round().astype(int).tolist()
    picks = sorted(set(edges + spread))
    rels = []
    for b_pick in range(B):
        sc_rows = sc[b_pick, picks].cpu()
        cpu = [x[b_pick:b_pick + 1].cpu() for x in args]
        # the oracle's causal rule needs each row's absolute position: row by row
        for j, tt in enumerate(picks):
            th1, id1, c1 = o.topk_select(sc_rows[j:j + 1], k, causal=True, rows_per_batch=1, q_row0=tt,
                                         idx_cap=cap)
            r = b_pick * T + tt
            assert th1[0] == thr[r].item()
            assert c1[0] == cnt[r].item()
            m = min(int(c1[0]), cap)
            assert np.array_equal(id1[0, :m], idx[r, :m].cpu().numpy())
            # indexer scores of the row vs the fp32 oracle (bf16 inputs upcast)
            ref = o.indexer_scores(*cpu[:3], slice(tt, tt + 1))[0, 0, : tt + 1]
            got = sc_rows[j, : tt + 1]
            mag = (cpu[0][0, tt].float().abs() @ cpu[1][0, : tt + 1].float().abs().T).mean().item()
            assert bool(((got - ref).abs() <= 2e-2 * ref.abs() + 1e-3 * mag).all())
            # attention of the row over the GPU's kept set (threshold form if the list overflowed)
            if int(cnt[r]) <= cap:
                oo = o.attention_from_lists(idx[r].cpu().numpy(), int(cnt[r]), *cpu[3:], 0, tt)
            else:
                oo = o.sparse_attention_with_threshold(sc[b_pick:b_pick + 1, tt:tt + 1].cpu(),
                                                       thr[r:r + 1].cpu().view(1, 1, 1), *cpu[3:],
                                                       rows=slice(tt, tt + 1))[0, 0]
            rels.append(assert_close_elementwise(O[b_pick, tt], oo, what=f"{name} row b={b_pick} t={tt}"))
    print(f"{name}: {len(rels)} sampled rows, max relative error of O {max(rels):.3e} "
          f"(|O| floored at {ATOL_16:g})")
