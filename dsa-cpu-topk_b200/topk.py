"""Per-row top-K threshold / kept-index selection on the GPU (stage 2).

GPU replacement of the reference's top-K code paths:

    topk_threshold(scores, k)              topk_avx512.cpp:251-253 (ext.topk_threshold)
    topk_threshold_batch_merge(scores, k)  topk_avx512.cpp:255-257 (same result, other CPU strategy)
    select_threshold(scores, top_k)        dsa_attention.py:41-44 / :343-344 (topk(...).values[..., -1:])
    topk_select(scores, k, ...)            threshold + ascending kept-index list + count

All run the radix-select kernel of libdsa_b200.so on the current stream; the
threshold equals torch.topk(scores, k).values[..., k-1] by value (-0.0 and
+0.0 are the same value), and the kept set is {s : scores[s] >= thr}
(ties kept), restricted to s <= t for causal rows.
"""
from __future__ import annotations

import torch

import _native


def idx_cap_for(k: int, row_len: int) -> int:
    """List capacity used by the forward: k plus room for ties, multiple of 32."""
    return min(row_len, ((k + k // 4 + 32 + 31) // 32) * 32)


def topk_select(scores: torch.Tensor, k: int, *, causal: bool = False, q_row0: int = 0,
                idx_cap: int | None = None, return_idx: bool = True):
    """scores [..., N] fp32 CUDA -> (thr [rows], idx [rows, idx_cap] int32, cnt [rows] int32).

    With ``causal`` the tensor must be [B, T_q, N]: row t (absolute position
    q_row0 + t) keeps only s <= t and entries s > t count as -inf.  Entries of
    idx past cnt (or all of it when return_idx is False) are unspecified /
    None.  cnt can exceed idx_cap when many values tie; then the list holds
    the first idx_cap kept positions.
    """
    assert scores.is_cuda and scores.dtype == torch.float32, "scores must be fp32 CUDA"
    N = scores.shape[-1]
    assert 1 <= k <= N, f"need 1 <= k <= N (k={k}, N={N})"
    s = _native.prep(scores)
    rows = s.numel() // N
    rows_per_batch = s.shape[-2] if (causal and s.dim() >= 2) else 1
    thr = torch.empty(rows, device=s.device, dtype=torch.float32)
    if not return_idx:
        _native.topk_select(s, rows, N, N, k, thr, causal=causal, rows_per_batch=rows_per_batch,
                            q_row0=q_row0)
        return thr, None, None
    cap = N if idx_cap is None else idx_cap
    idx = torch.empty((rows, cap), device=s.device, dtype=torch.int32)
    cnt = torch.empty(rows, device=s.device, dtype=torch.int32)
    _native.topk_select(s, rows, N, N, k, thr, idx, cnt, cap, causal=causal,
                        rows_per_batch=rows_per_batch, q_row0=q_row0)
    return thr, idx, cnt


def topk_select_bitmap(scores: torch.Tensor, k: int, *, causal: bool = True, q_row0: int = 0,
                       workspace: bool = True):
    """scores [B, T_q, N] fp32 CUDA -> (thr [rows], cnt [rows] int32, bits [rows, words] int32).

    The kept set of each row (score >= thr, and s <= q_row0 + t when causal)
    as the bitmap of dsa_attention.kept_bitmap, written by the top-K kernels
    themselves where the row length allows (4K-32K entries).  workspace=True
    gives them a candidate workspace (the sweep + resolve kernels); False runs
    the one-kernel form that needs none."""
    assert scores.is_cuda and scores.dtype == torch.float32 and scores.dim() == 3, \
        "scores must be fp32 CUDA [B, T_q, N]"
    B, T_q, N = scores.shape
    assert 1 <= k <= N, f"need 1 <= k <= N (k={k}, N={N})"
    s = _native.prep(scores)
    thr = torch.empty(B * T_q, device=s.device, dtype=torch.float32)
    cnt = torch.empty(B * T_q, device=s.device, dtype=torch.int32)
    bits = torch.empty((B * T_q, _native.bitmap_words(N)), device=s.device, dtype=torch.int32)
    ws = None
    if workspace:
        ws = torch.empty(_native.topk_select_bitmap_workspace_bytes(B * T_q, bits.shape[-1]),
                         device=s.device, dtype=torch.uint8)
    _native.topk_select_bitmap(s, k, thr, bits, cnt, causal=causal, q_row0=q_row0, workspace=ws)
    return thr, cnt, bits


def topk_threshold(scores: torch.Tensor, k: int) -> torch.Tensor:
    """[..., N] fp32 -> [..., 1] k-th largest per row (topk_avx512.cpp:226-253 contract)."""
    assert k > 0, "k must be > 0"
    assert k <= scores.shape[-1], "k must be <= N"
    thr, _, _ = topk_select(scores, k, return_idx=False)
    return thr.view(*scores.shape[:-1], 1)


def topk_threshold_batch_merge(scores: torch.Tensor, k: int) -> torch.Tensor:
    """Same result as topk_threshold (the reference's second CPU strategy)."""
    return topk_threshold(scores, k)


def select_threshold(scores: torch.Tensor, top_k: int) -> torch.Tensor:
    """dsa_attention.py:41-44: k_eff = min(top_k, N); returns thr [..., 1]."""
    return topk_threshold(scores, min(top_k, scores.shape[-1]))


if __name__ == "__main__":
    # Timing driver for the forward's bitmap top-K: causal rows of N(0,1)
    # scores [B, T, T], k per row, the sweep + resolve kernels (workspace)
    # checked bit for bit against the one-kernel form, then timed with CUDA
    # events, L2 flushed between runs.
    import argparse

    ap = argparse.ArgumentParser(description="time topk_select_bitmap on causal N(0,1) rows")
    ap.add_argument("--B", type=int, default=1)
    ap.add_argument("--T", type=int, default=32768)
    ap.add_argument("--k", type=int, default=2048)
    ap.add_argument("--runs", type=int, default=10)
    ap.add_argument("--zigzag", default=None, metavar="N:r",
                    help="only the rows rank r of N owns under the zig-zag split of one sequence "
                         "(two row blocks, one call with row_bstep)")
    args = ap.parse_args()
    g = torch.Generator(device="cuda").manual_seed(0)
    if args.zigzag:
        from sharding import zigzag_plan
        n, r = (int(x) for x in args.zigzag.split(":"))
        b0, b1 = zigzag_plan(args.T, n)[r]
        assert b0.stop - b0.start == b1.stop - b1.start, "zig-zag blocks of equal rows"
        s = torch.randn((2, b0.stop - b0.start, args.T), device="cuda", generator=g)
        q_row0, bstep = b0.start, b1.start - b0.start
    else:
        s = torch.randn((args.B, args.T, args.T), device="cuda", generator=g)
        q_row0, bstep = 0, 0
    B_, T_q, N = s.shape
    words = _native.bitmap_words(N)

    def run(ws):
        thr = torch.empty(B_ * T_q, device="cuda", dtype=torch.float32)
        cnt = torch.empty(B_ * T_q, device="cuda", dtype=torch.int32)
        bits = torch.empty((B_ * T_q, words), device="cuda", dtype=torch.int32)
        _native.topk_select_bitmap(s, args.k, thr, bits, cnt, causal=True, q_row0=q_row0, row_bstep=bstep,
                                   workspace=ws)
        return thr, cnt, bits

    ws = torch.empty(_native.topk_select_bitmap_workspace_bytes(B_ * T_q, words), device="cuda",
                     dtype=torch.uint8)
    if bstep == 0:
        one = run(None)
        two = run(ws)
        assert all(torch.equal(x, y) for x, y in zip(one, two)), "sweep + resolve differs from the one-kernel form"
    flush = torch.empty(256 << 20, device="cuda", dtype=torch.uint8)
    ts = []
    for i in range(args.runs + 2):
        flush.zero_()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        run(ws)
        e1.record()
        torch.cuda.synchronize()
        ts.append(e0.elapsed_time(e1))
    ts = sorted(ts[2:])
    print(f"topk_select_bitmap B={B_} T_q={T_q} N={N} k={args.k} zigzag={args.zigzag}: "
          f"min {ts[0]:.3f} ms, median {ts[len(ts) // 2]:.3f} ms")
