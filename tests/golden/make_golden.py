"""Generate the golden fixtures in tests/golden/ from the reference itself.

Run once, in a container where the reference checkout is mounted:

    python tests/golden/make_golden.py [REFERENCE_DIR]

It imports the reference's own torch functions (lightning_indexer.py,
dsa_attention.py) and its AVX-512 top-K extension (topk_avx512.cpp, built by
oracle/build_ref.py) and records their outputs on seeded CPU inputs.  The
reference's tests seed a CUDA generator (test_dsa.py:12-14,
test_indexer.py:12-14) which a CPU cannot reproduce, so the same shapes are
drawn here from CPU generators instead; the inputs are stored in the
fixtures, so nothing needs the reference at test time.

Shapes follow the reference tests:
  indexer_*.npz   test_indexer.py:18-33 shapes (1,64,4,64) (2,128,8,64) (1,200,4,32)
  project.npz     test_indexer.py:36-48 (B=2,T=96,D=128,H=4,d=64)
  topk_*.npz      test_topk_avx512.py:20-35 (randn(3,128,128), k in 1..128) plus tie cases
  dsa_*.npz       test_dsa.py:27-61 shapes, a non-power-of-2 T, a bf16 case and
                  one batch of config c1 (T=512, k=32)
"""
from __future__ import annotations

import math
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))


def rnd(shape, seed, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(shape, generator=g, dtype=torch.float32) * scale


def save(name, **arrays):
    path = os.path.join(HERE, name + ".npz")
    np.savez_compressed(path, **{k: (v.numpy() if isinstance(v, torch.Tensor) else np.asarray(v))
                                 for k, v in arrays.items()})
    print(f"{name}.npz  {os.path.getsize(path)/1024:.0f} KB")


def main(ref_dir):
    sys.path.insert(0, ref_dir)
    import lightning_indexer as li  # noqa: E402  (reference)
    import dsa_attention as da      # noqa: E402  (reference)
    sys.path.insert(0, os.path.join(REPO, "oracle"))
    import build_ref                # noqa: E402
    build_ref.build(ref_dir)
    ext = build_ref.load_ref()
    assert ext is not None, "reference AVX-512 top-K did not build"

    torch.set_num_threads(max(1, os.cpu_count() or 1))

    # ---- indexer scores (test_indexer.py:18-33) ----
    for (B, T, H, d) in [(1, 64, 4, 64), (2, 128, 8, 64), (1, 200, 4, 32)]:
        q, k, w = rnd((B, T, H, d), 0), rnd((B, T, d), 1), rnd((B, T, H), 2)
        save(f"indexer_B{B}_T{T}_H{H}_d{d}", q=q, k=k, w=w,
             scores=li.indexer_scores_torch(q, k, w),
             mask8=li.topk_mask(li.indexer_scores_torch(q, k, w), 8))

    # ---- projection front-end (test_indexer.py:36-48) ----
    B, T, D, H, d = 2, 96, 128, 4, 64
    h = rnd((B, T, D), 0)
    W_Q, W_K, W_W = rnd((D, H * d), 10, 0.1), rnd((D, d), 11, 0.1), rnd((D, H), 12, 0.1)
    save("project", h=h, W_Q=W_Q, W_K=W_K, W_W=W_W, H=H, d=d,
         scores=li.indexer_torch(h, W_Q, W_K, W_W, H, d))

    # ---- top-K thresholds (test_topk_avx512.py:20-35) ----
    torch.manual_seed(0)
    x = torch.randn(3, 128, 128, dtype=torch.float32)
    ks = np.array([1, 8, 16, 32, 64, 96, 128])
    thr_torch = np.stack([x.topk(int(kk), dim=-1).values[..., -1].numpy() for kk in ks])
    thr_avx = np.stack([ext.topk_threshold(x.contiguous(), int(kk))[..., 0].numpy() for kk in ks])
    thr_bm = np.stack([ext.topk_threshold_batch_merge(x.contiguous(), int(kk))[..., 0].numpy()
                       for kk in ks])
    assert np.array_equal(thr_torch, thr_avx) and np.array_equal(thr_torch, thr_bm)
    save("topk_randn", x=x, ks=ks, thr=thr_torch)

    # tie-heavy rows: quantised values, exact zeros of both signs, all-equal rows,
    # -inf tails (causal masking), and rows of exactly k finite entries.
    g = torch.Generator().manual_seed(7)
    rows = []
    rows.append(torch.round(torch.randn(16, 256, generator=g) * 2) / 2)          # few distinct values
    z = torch.randn(16, 256, generator=g)
    z[z.abs() < 0.8] = 0.0
    z[:, ::3] = torch.where(z[:, ::3] == 0, torch.tensor(-0.0), z[:, ::3])      # -0.0 mixed with +0.0
    rows.append(z)
    rows.append(torch.full((4, 256), 1.25))                                      # all equal
    rows.append(torch.zeros(4, 256))                                             # all zero
    m = torch.randn(16, 256, generator=g)
    for r in range(16):
        m[r, 8 * r + 1:] = float("-inf")                                         # causal-style tails
    rows.append(m)
    rows.append(torch.full((2, 256), float("-inf")))                             # all -inf
    xt = torch.cat(rows).contiguous()
    kt = np.array([1, 4, 16, 32, 64, 128, 256])
    thr_t = np.stack([xt.topk(int(kk), dim=-1).values[..., -1].numpy() for kk in kt])
    thr_ta = np.stack([ext.topk_threshold(xt, int(kk))[..., 0].numpy() for kk in kt])
    # the reference extension is built with -ffast-math; record whether it agrees
    save("topk_ties", x=xt, ks=kt, thr=thr_t, thr_avx512=thr_ta,
         avx512_agrees=np.array([np.array_equal(a, b) for a, b in zip(thr_t, thr_ta)]))

    # ---- DSA forward (test_dsa.py) ----
    def dsa_case(name, B, T, HI, DI, HQ, DQ, DV, top_k, scale=0.3, dtype=torch.float32,
                 w_scale=None, v_scale=1.0, naive=False):
        qi = (rnd((B, T, HI, DI), 0, scale)).to(dtype)
        ki = (rnd((B, T, DI), 1, scale)).to(dtype)
        wi = rnd((B, T, HI), 2, scale if w_scale is None else w_scale)
        Q = (rnd((B, T, HQ, DQ), 3, scale)).to(dtype)
        K = (rnd((B, T, HQ, DQ), 4, scale)).to(dtype)
        V = (rnd((B, T, HQ, DV), 5, v_scale)).to(dtype)
        f = [t.float() for t in (qi, ki, wi, Q, K, V)]
        out = da.dsa_attention_torch(*f, top_k=top_k)
        scores = li.indexer_scores_torch(*f[:3])
        thr = scores.topk(min(top_k, T), dim=-1).values[..., -1:]
        arrays = dict(q_idx=f[0], k_idx=f[1], w_idx=f[2], Q=f[3], K=f[4], V=f[5],
                      top_k=top_k, out=out, thr=thr, dtype=str(dtype).split(".")[-1])
        if naive:
            arrays["out_naive"] = da.dsa_attention_naive(*f, top_k=top_k)
        save(name, **arrays)

    dsa_case("dsa_naive_T16", 1, 16, 2, 16, 2, 16, 16, 4, naive=True)
    dsa_case("dsa_small_B2_T32", 2, 32, 2, 16, 2, 16, 16, 8, naive=True)
    for T, kk in [(32, 8), (64, 16), (128, 32)]:
        dsa_case(f"dsa_T{T}_k{kk}", 1, T, 4, 32, 4, 32, 32, kk)
    dsa_case("dsa_T200_k24", 2, 200, 4, 32, 4, 32, 32, 24)                 # non-power-of-2 T
    dsa_case("dsa_c1_B1", 1, 512, 4, 32, 4, 32, 32, 32, scale=1.0,
             w_scale=1 / math.sqrt(4))                                       # config c1, one batch
    dsa_case("dsa_bf16_T256", 1, 256, 4, 64, 4, 64, 64, 16, scale=1.0,
             dtype=torch.bfloat16, w_scale=1 / math.sqrt(4))


if __name__ == "__main__":
    ref = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("DSA_REFERENCE_DIR")
    if not ref:
        sys.exit("usage: make_golden.py <reference checkout> (or set DSA_REFERENCE_DIR)")
    main(ref)
