"""The reference's hybrid entry point, served entirely on the GPU.

The reference (dsa_hybrid.py:36-66) runs the indexer on the GPU, copies the
[B,T,T] score matrix to pinned host memory, finds each row's k-th largest
with AVX-512 on the CPU, copies the thresholds back and runs the
threshold-form attention.  On B200 that round trip is pure overhead: the
radix-select top-K runs on the device between the other two stages.

``HybridContext`` keeps its role of holding reusable buffers across calls
(here: the device workspace of the three-stage pipeline), and
``dsa_hybrid_cpu_topk`` keeps its signature, so existing callers run
unchanged; the result equals dsa_attention_split_triton's.
"""
from __future__ import annotations

import torch

import dsa_attention


class HybridContext:
    """Reusable device workspace for [B, T] forwards."""

    def __init__(self, B, T, top_k: int | None = None, device=None):
        self.B, self.T = B, T
        self.device = torch.device("cuda") if device is None else torch.device(device)
        self._ws = None
        if top_k is not None:
            self.workspace(top_k)

    def workspace(self, top_k: int) -> torch.Tensor:
        need = dsa_attention.forward_workspace_bytes(self.B, self.T, self.T, top_k)
        if self._ws is None or self._ws.numel() < need:
            self._ws = torch.empty(need, device=self.device, dtype=torch.uint8)
        return self._ws


def dsa_hybrid_cpu_topk(q_idx, k_idx, w_idx, Q, K, V, top_k: int,
                        ctx: HybridContext | None = None) -> torch.Tensor:
    B, T = Q.shape[0], Q.shape[1]
    if ctx is None:
        ctx = HybridContext(B, T, device=Q.device)
    assert ctx.B == B and ctx.T == T
    assert 0 < top_k <= T
    return dsa_attention.dsa_forward(q_idx, k_idx, w_idx, Q, K, V, top_k,
                                     workspace=ctx.workspace(top_k))
