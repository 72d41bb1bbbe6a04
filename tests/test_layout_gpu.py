"""GPU: strided inputs and row blocks through the _ex entry points.

The kernels read every input through its strides (tensor maps on the tensor
cores, pointer arithmetic elsewhere), so a strided view must give the same
bits as its contiguous copy.  Row blocks of one sequence run in one launch
per stage (batch b of the query side at rows q_row0 + b*row_bstep, the key
side shared with batch stride 0) and must give the same bits as separate
calls and as the whole forward: each query row is computed independently
(dsa_attention.py:213, :312, the reference's per-query grid)."""
import pytest
import torch

import dsa_oracle as o

pytestmark = pytest.mark.gpu

SHAPES = [
    # B, T, HI, DI, HQ, D, k, dtype   (tensor-core indexer + attention / CUDA cores + gather)
    (1, 1024, 8, 128, 4, 128, 64, torch.bfloat16),
    (2, 640, 4, 64, 2, 64, 48, torch.bfloat16),
    (2, 300, 4, 32, 4, 32, 32, torch.float32),
]


@pytest.mark.parametrize("B,T,HI,DI,HQ,D,k,dtype", SHAPES)
def test_strided_views_equal_contiguous(cuda, B, T, HI, DI, HQ, D, k, dtype):
    """K/V sliced from a fused [B, T, 3, HQ, D] projection, q_idx sliced from
    wider heads, w from a padded buffer: no copies, identical output."""
    from dsa_attention import dsa_forward
    qi, ki, wi, Q, K, V = (x.to(cuda) for x in o.make_inputs(B, T, HI, DI, HQ, D, D, dtype=dtype))
    whole = dsa_forward(qi, ki, wi, Q, K, V, k)
    qkv = torch.stack([Q, K, V], dim=2)                        # [B, T, 3, HQ, D]
    q_big = torch.zeros(B, T, HI + 3, DI, device=cuda, dtype=dtype)
    q_big[:, :, 1:HI + 1] = qi
    w_big = torch.zeros(B, T, HI + 4, device=cuda)
    w_big[:, :, :HI] = wi
    k_big = torch.zeros(B, T, 2 * DI, device=cuda, dtype=dtype)
    k_big[:, :, DI:] = ki
    views = (q_big[:, :, 1:HI + 1], k_big[:, :, DI:], w_big[:, :, :HI], qkv[:, :, 0], qkv[:, :, 1],
             qkv[:, :, 2])
    assert not any(v.is_contiguous() for v in views)
    out = dsa_forward(*views, k)
    assert torch.equal(out, whole)


@pytest.mark.parametrize("B,T,HI,DI,HQ,D,k,dtype", SHAPES)
@pytest.mark.parametrize("world", [2, 4])
def test_zigzag_row_blocks_in_one_call(cuda, B, T, HI, DI, HQ, D, k, dtype, world):
    """Every rank's two zig-zag blocks (r and 2N-1-r) in ONE forward call equal
    the same rows of the whole forward, bit for bit."""
    import sharding
    from dsa_attention import dsa_forward
    T = (T // (2 * world)) * (2 * world)
    qi, ki, wi, Q, K, V = (x.to(cuda) for x in o.make_inputs(B, T, HI, DI, HQ, D, D, dtype=dtype))
    whole = dsa_forward(qi, ki, wi, Q, K, V, k)
    for r, blocks in enumerate(sharding.zigzag_plan(T, world)):
        a, b = blocks
        n = a.stop - a.start
        assert b.stop - b.start == n
        for bb in range(B):
            pick = lambda x: torch.stack([x[bb, a.start:a.stop], x[bb, b.start:b.stop]])
            out = dsa_forward(pick(qi), ki[bb:bb + 1], pick(wi), pick(Q), K[bb:bb + 1], V[bb:bb + 1], k,
                              q_row0=a.start, row_bstep=b.start - a.start)
            assert torch.equal(out[0], whole[bb, a.start:a.stop]), f"rank {r} batch {bb} low block"
            assert torch.equal(out[1], whole[bb, b.start:b.stop]), f"rank {r} batch {bb} high block"


def test_indexer_and_topk_row_blocks(cuda):
    """Stage by stage: scores and selections of row blocks in one call equal
    the per-block calls (tensor-core indexer, bitmap top-K with row_bstep)."""
    import _native
    from lightning_indexer import indexer_scores
    from topk import topk_select_bitmap
    B, T, HI, DI, k = 1, 4096, 8, 128, 256
    qi, ki, wi, _, _, _ = (x.to(cuda) for x in o.make_inputs(B, T, HI, DI, 1, 16, 16, dtype=torch.bfloat16))
    blocks = [(256, 768), (3072, 3584)]
    stack = lambda x: torch.cat([x[:, a:z] for a, z in blocks])
    sc = indexer_scores(stack(qi), ki, stack(wi), q_row0=256, row_bstep=3072 - 256, fill_upper=False)
    n = 512
    for i, (a, z) in enumerate(blocks):
        ref = indexer_scores(qi[:, a:z], ki, wi[:, a:z], q_row0=a, fill_upper=False)
        causal = torch.arange(T, device=cuda).view(1, T) <= torch.arange(a, z, device=cuda).view(n, 1)
        assert torch.equal(sc[i][causal], ref[0][causal])
    rows = 2 * n
    thr = torch.empty(rows, device=cuda)
    cnt = torch.empty(rows, device=cuda, dtype=torch.int32)
    bits = torch.empty(rows, _native.bitmap_words(T), device=cuda, dtype=torch.int32)
    _native.topk_select_ex(sc, rows, T, T, k, thr, None, cnt, 0, bits, causal=True, rows_per_batch=n,
                           q_row0=256, row_bstep=3072 - 256)
    for i, (a, z) in enumerate(blocks):
        t1, c1, b1 = topk_select_bitmap(sc[i:i + 1], k, q_row0=a)
        assert torch.equal(thr[i * n:(i + 1) * n], t1)
        assert torch.equal(cnt[i * n:(i + 1) * n], c1)
        assert torch.equal(bits[i * n:(i + 1) * n], b1)


def test_non_16_byte_strides_take_the_cuda_core_path(cuda):
    """A stride that is not a multiple of 16 bytes cannot feed a tensor map:
    the wrapper copies such an input (same result), and the C ABI reports it
    for the tensor-core-only entry point."""
    import _native
    from dsa_attention import dsa_forward
    B, T, HI, DI, HQ, D, k = 1, 256, 3, 64, 2, 64, 32
    qi, ki, wi, Q, K, V = (x.to(cuda) for x in o.make_inputs(B, T, HI, DI, HQ, D, D, dtype=torch.bfloat16))
    whole = dsa_forward(qi, ki, wi, Q, K, V, k)
    kpad = torch.zeros(B, T, DI + 1, device=cuda, dtype=torch.bfloat16)   # row stride 130 bytes
    kpad[:, :, :DI] = ki
    assert torch.equal(dsa_forward(qi, kpad[:, :, :DI], wi, Q, K, V, k), whole)
    Vpad = torch.zeros(B, T, HQ, D + 8, device=cuda, dtype=torch.bfloat16)  # head stride 144 bytes
    Vpad[..., :D] = V
    bits = torch.zeros(B * T, _native.bitmap_words(T), device=cuda, dtype=torch.int32)
    O = torch.empty(B, T, HQ, D, device=cuda)
    _native.sparse_attn_bitmap_ex(bits, Q, K, Vpad[..., :D], O)            # 144-byte stride: allowed
    Vodd = torch.zeros(B, T, HQ, D + 1, device=cuda, dtype=torch.bfloat16)  # 130 bytes: not
    with pytest.raises(RuntimeError, match="stride"):
        _native.sparse_attn_bitmap_ex(bits, Q, K, Vodd[..., :D], O)
