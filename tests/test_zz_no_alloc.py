"""GPU: dsa_forward_noalloc, the forward for callers that cannot allocate.

Some callers cannot call cudaMalloc where they run the forward: a host
framework that owns every byte of GPU memory through its own pool, or a
plugin that is only handed its input and output buffers.  They cannot
provide dsa_forward's workspace, so dsa_forward_noalloc keeps that workspace
in a fixed 32 MiB array inside the library.

The test calls it through the C ABI (the ctypes binding in _native.py) and
checks its output against dsa_forward's (the caller-workspace entry point)
on two calls in a row with different data.  Both run the same kernels on the
same inputs into same-layout workspaces, so the outputs must be equal bit
for bit: a stale or partly reused scratch region would show up.  Cases cover
a row block at an offset (q_row0 > 0, T_q < T_k) and bf16 heads of 64, and a
shape needing more than 32 MiB is refused.  The file creates all of its own
inputs and passes both alone in a fresh process and after the other tests;
it is named so that pytest collects it last.
"""
import pytest
import torch

import dsa_oracle as o

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("B,T,HI,DI,HQ,D,k,dtype,q_row0,T_q", [
    (16, 512, 4, 32, 4, 32, 32, torch.float32, 0, 512),        # config c1 (fits in the 32 MiB)
    (1, 1024, 8, 128, 16, 128, 96, torch.bfloat16, 0, 1024),   # tensor-core indexer and attention
    (2, 1024, 4, 64, 8, 64, 64, torch.bfloat16, 600, 300),     # row block at an offset, D = 64
])
def test_noalloc_matches_dsa_forward_twice(cuda, B, T, HI, DI, HQ, D, k, dtype, q_row0, T_q):
    import _native
    from dsa_attention import dsa_forward
    rows = slice(q_row0, q_row0 + T_q)
    for seed in (0, 100):  # two calls in a row, different data
        qi, ki, wi, Q, K, V = (x.to(cuda).contiguous() for x in
                               o.make_inputs(B, T, HI, DI, HQ, D, D, dtype=dtype, seed0=seed))
        qi, wi, Q = (x[:, rows].contiguous() for x in (qi, wi, Q))
        ref = dsa_forward(qi, ki, wi, Q, K, V, k, q_row0=q_row0)
        O = torch.full((B, T_q, HQ, D), float("nan"), device=cuda, dtype=torch.float32)
        _native.forward_noalloc(qi, ki, wi, Q, K, V, O, k, q_row0=q_row0)
        torch.cuda.synchronize()
        assert torch.isfinite(O).all()
        assert torch.equal(O, ref), f"seed {seed}: max diff {(O - ref).abs().max().item()}"


def test_noalloc_rejects_shapes_beyond_its_scratch(cuda):
    import _native
    args = [x.to(cuda) for x in o.make_inputs(1, 4096, 1, 16, 1, 16, 16)]
    O = torch.empty((1, 4096, 1, 16), device=cuda)
    with pytest.raises(AssertionError, match="scratch"):   # 4096 x 4096 fp32 scores alone are 64 MiB
        _native.forward_noalloc(*args, O, 64)
