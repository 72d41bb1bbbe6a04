"""Query-row sharding of the DSA forward across GPUs (one process per GPU).

Query row t of a sequence depends only on its own q_idx / w_idx / Q rows and
on the key-side rows s <= t (k_idx, K, V), so the forward shards by
(batch x query-row block) with no exchange: every rank holds the full
key-side tensors of its batches and computes its own rows.  The reference
has no multi-GPU code; this is the B200 design's partitioning.

Causal cost grows with t, so a plan cuts each sequence into 2*N blocks and
gives rank r blocks r and 2N-1-r ("zig-zag"): every rank then gets the same
number of rows and nearly the same number of (t, s) pairs.

NCCL is used only after the forward, to gather output rows for verification
(``gather_rows``); nothing on the hot path communicates.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class RowBlock:
    start: int  # absolute query row of the block's first row
    stop: int   # one past the last row


def zigzag_plan(T: int, world: int) -> list[list[RowBlock]]:
    """Row blocks of each rank: rank r owns blocks r and 2*world-1-r of 2*world."""
    assert T >= 1 and world >= 1
    nb = 2 * world
    edges = [(T * i) // nb for i in range(nb + 1)]
    blocks = [RowBlock(edges[i], edges[i + 1]) for i in range(nb)]
    return [[blocks[r], blocks[nb - 1 - r]] for r in range(world)]


def causal_pairs(blocks: list[RowBlock], T_k: int | None = None) -> int:
    """Number of causal (t, s) pairs of the given rows: sum of min(t+1, T_k)."""
    n = 0
    for b in blocks:
        a, z = b.start, b.stop
        if T_k is None or z <= T_k:
            n += (z * (z + 1) - a * (a + 1)) // 2
        else:
            n += sum(min(t + 1, T_k) for t in range(a, z))
    return n


def forward_rows(forward, q_idx, k_idx, w_idx, Q, K, V, top_k, blocks: list[RowBlock], **kw):
    """Run ``forward`` (dsa_attention.dsa_forward-compatible) on each row block.

    The query-side tensors hold all T rows; the key side is shared.  Returns
    the output rows of the blocks, concatenated in block order.
    """
    outs = []
    for b in blocks:
        if b.stop > b.start:
            outs.append(forward(q_idx[:, b.start:b.stop], k_idx, w_idx[:, b.start:b.stop],
                                Q[:, b.start:b.stop], K, V, top_k, q_row0=b.start, **kw))
    return torch.cat(outs, dim=1)


def gather_rows(local: torch.Tensor, plan: list[list[RowBlock]], group=None) -> torch.Tensor:
    """All-gather every rank's output rows and reassemble them in row order.

    local: [B, rows_of_this_rank, ...] in the rank's block order.  Works with
    any torch.distributed backend (NCCL on GPUs, gloo on CPU).
    """
    import torch.distributed as dist
    world = dist.get_world_size(group)
    sizes = [sum(b.stop - b.start for b in plan[r]) for r in range(world)]
    width = max(sizes)
    pad = torch.zeros((local.shape[0], width) + tuple(local.shape[2:]), dtype=local.dtype,
                      device=local.device)
    pad[:, : local.shape[1]] = local
    bufs = [torch.empty_like(pad) for _ in range(world)]
    dist.all_gather(bufs, pad, group=group)
    T = max(b.stop for r in plan for b in r)
    out = torch.empty((local.shape[0], T) + tuple(local.shape[2:]), dtype=local.dtype,
                      device=local.device)
    for r in range(world):
        off = 0
        for b in plan[r]:
            n = b.stop - b.start
            out[:, b.start:b.stop] = bufs[r][:, off:off + n]
            off += n
    return out
