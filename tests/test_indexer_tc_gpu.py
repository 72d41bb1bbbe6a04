"""GPU: the tcgen05 tensor-core indexer (bf16, DI in {64, 128}) against the
fp32 CUDA-core kernel and the oracle, on ragged shapes.

Both GPU kernels compute from identical bf16 inputs; they differ only in
fp32 summation order, so they agree to ~1e-5 relative; the oracle (fp32
einsum of the upcast inputs) to rtol 2e-2 (the bf16 parity bar), in practice
far tighter."""
import os

import pytest
import torch

import dsa_oracle as o

pytestmark = pytest.mark.gpu


def scores(q, k, w, **kw):
    from lightning_indexer import indexer_scores
    return indexer_scores(q, k, w, **kw)


def simt_scores(q, k, w, **kw):
    os.environ["DSA_FORCE_SIMT_INDEXER"] = "1"
    try:
        return scores(q, k, w, **kw)
    finally:
        del os.environ["DSA_FORCE_SIMT_INDEXER"]


@pytest.mark.parametrize("B,T_q,T_k,q0,HI,DI", [
    (1, 256, 256, 0, 4, 64),
    (1, 300, 300, 0, 3, 128),       # ragged query and key blocks
    (2, 1000, 1000, 0, 16, 64),
    (1, 129, 1001, 872, 8, 128),    # row block at an offset, T_k % 4 != 0
    (3, 1, 513, 512, 2, 64),        # single query row
    (1, 2048, 2048, 0, 64, 128),    # c5 head shapes
    # TMA score stores (T_k % 4 == 0) at row offsets with several batches:
    # ragged T_q (rows past it clipped at the batch edge) and a partial last chunk
    (2, 200, 1004, 804, 4, 64),
    (2, 72, 1028, 956, 8, 128),
])
def test_tc_matches_simt_and_oracle(cuda, B, T_q, T_k, q0, HI, DI):
    g = torch.Generator().manual_seed(T_q + 7 * HI)
    q = torch.randn(B, T_q, HI, DI, generator=g).bfloat16()
    k = torch.randn(B, T_k, DI, generator=g).bfloat16()
    w = torch.randn(B, T_q, HI, generator=g) / HI ** 0.5
    dq, dk, dw = q.to(cuda), k.to(cuda), w.to(cuda)
    tc = scores(dq, dk, dw, q_row0=q0).cpu()
    sm = simt_scores(dq, dk, dw, q_row0=q0).cpu()
    fin = torch.isfinite(sm)
    assert torch.equal(torch.isfinite(tc), fin)
    assert torch.isneginf(tc[~fin]).all()
    err = (tc[fin] - sm[fin]).abs()
    scale = torch.einsum("bthd,bsd->bts", q.float().abs(), k.float().abs()).mean().item()
    assert err.max().item() < 1e-5 * scale * HI ** 0.5 + 1e-6, err.max().item()
    # oracle on the absolute rows
    qf = torch.zeros(B, q0 + T_q, HI, DI)
    wf = torch.zeros(B, q0 + T_q, HI)
    qf[:, q0:], wf[:, q0:] = q.float(), w
    kf = k.float()
    if kf.shape[1] < qf.shape[1]:
        kf = torch.cat([kf, torch.zeros(B, qf.shape[1] - kf.shape[1], DI)], 1)
    ref = o.indexer_scores(qf, kf, wf, slice(q0, q0 + T_q), T_k=T_k)
    assert torch.equal(torch.isfinite(ref), fin)
    e2 = (tc[fin] - ref[fin]).abs()
    assert bool((e2 <= 2e-2 * ref[fin].abs() + 1e-4 * scale).all()), e2.max().item()


def test_tc_fill_upper_contract(cuda):
    q = torch.randn(1, 384, 4, 64).bfloat16().to(cuda)
    k = torch.randn(1, 384, 64).bfloat16().to(cuda)
    w = torch.randn(1, 384, 4).to(cuda)
    full = scores(q, k, w, fill_upper=True)
    upper = ~torch.ones(384, 384, dtype=torch.bool, device=cuda).tril()
    assert torch.isneginf(full[0][upper]).all()
    part = scores(q, k, w, fill_upper=False)
    assert torch.equal(part[0][~upper], full[0][~upper])


@pytest.mark.parametrize("B,T_q,T_k,q0,HI,DI", [
    (1, 300, 300, 0, 4, 128),
    (2, 700, 700, 0, 8, 128),
    (1, 129, 1001, 872, 2, 256),
    (1, 2048, 2048, 0, 64, 128),     # c5 head shapes
])
def test_fp8_tc_matches_simt_and_oracle(cuda, B, T_q, T_k, q0, HI, DI):
    """FP8 (e4m3) indexer inputs on the tensor cores (kind::f8f6f4).  Products
    of e4m3 values are exact in fp32, so the scores match the fp32 oracle on
    the upcast inputs to fp32 rounding."""
    g = torch.Generator().manual_seed(T_q + HI)
    q8 = (torch.randn(B, T_q, HI, DI, generator=g) * 2).to(torch.float8_e4m3fn)
    k8 = (torch.randn(B, T_k, DI, generator=g) * 2).to(torch.float8_e4m3fn)
    w = torch.randn(B, T_q, HI, generator=g) / HI ** 0.5
    dq, dk, dw = q8.to(cuda), k8.to(cuda), w.to(cuda)
    tc = scores(dq, dk, dw, q_row0=q0).cpu()
    sm = simt_scores(dq, dk, dw, q_row0=q0).cpu()
    fin = torch.isfinite(sm)
    assert torch.equal(torch.isfinite(tc), fin)
    qf, kf = q8.float(), k8.float()
    scale = torch.einsum("bthd,bsd->bts", qf.abs(), kf.abs()).mean().item()
    assert (tc[fin] - sm[fin]).abs().max().item() < 1e-5 * scale * HI ** 0.5 + 1e-6
    qfull = torch.zeros(B, q0 + T_q, HI, DI)
    wfull = torch.zeros(B, q0 + T_q, HI)
    qfull[:, q0:], wfull[:, q0:] = qf, w
    if kf.shape[1] < qfull.shape[1]:
        kf = torch.cat([kf, torch.zeros(B, qfull.shape[1] - kf.shape[1], DI)], 1)
    ref = o.indexer_scores(qfull, kf, wfull, slice(q0, q0 + T_q), T_k=T_k)
    assert bool(((tc[fin] - ref[fin]).abs() <= 1e-3 * ref[fin].abs() + 1e-5 * scale).all())


def test_fp8_indexer_in_forward(cuda):
    """Forward with FP8 indexer inputs and bf16 attention inputs, against the
    oracle run on the upcast values."""
    from dsa_attention import dsa_forward
    B, T, HI, DI, HQ, D, k = 1, 1024, 8, 128, 4, 64, 64
    qi, ki, wi, Q, K, V = o.make_inputs(B, T, HI, DI, HQ, D, D, dtype=torch.bfloat16)
    qi8, ki8 = qi.float().to(torch.float8_e4m3fn), ki.float().to(torch.float8_e4m3fn)
    out = dsa_forward(qi8.to(cuda), ki8.to(cuda), wi.to(cuda), Q.to(cuda), K.to(cuda), V.to(cuda), k).cpu()
    ref = o.dsa_attention(qi8.float(), ki8.float(), wi, Q, K, V, k)
    bad = ((out - ref).abs() > 2e-2 * ref.abs() + 2e-2).any(-1).any(-1)
    assert bad.float().mean() < 0.002


@pytest.mark.parametrize("B,T,HI,DI", [(1, 640, 8, 128), (2, 300, 4, 256), (1, 200, 4, 64)])
def test_fp8_indexer_with_row_scales_matches_dequantised_oracle(cuda, B, T, HI, DI):
    """Per-row e4m3 quantisation with the key scales applied to the score
    columns and the query scales folded into w: equal, to fp32 rounding, to the
    fp32 oracle on the dequantised inputs (products of e4m3 values are exact),
    on the tensor cores (DI 128/256) and on the CUDA cores (DI 64)."""
    from lightning_indexer import indexer_scores_fp8, quantize_fp8
    g = torch.Generator().manual_seed(T + DI)
    q = (torch.randn(B, T, HI, DI, generator=g) * 3).to(cuda)
    k = (torch.randn(B, T, DI, generator=g) * 0.01).to(cuda)        # scales far from 1
    w = (torch.randn(B, T, HI, generator=g) / HI ** 0.5).to(cuda)
    out = indexer_scores_fp8(q, k, w).cpu()
    q8, qs = quantize_fp8(q)
    k8, ks = quantize_fp8(k)
    assert q8.dtype == torch.float8_e4m3fn and bool((qs > 0).all())
    qd = (q8.float() * qs[..., None]).cpu()
    kd = (k8.float() * ks[..., None]).cpu()
    # e4m3: 3 mantissa bits (relative error <= 2^-4), subnormal steps of 2^-9 * scale
    assert bool(((qd - q.cpu()).abs() <= 0.0625 * q.cpu().abs() + 2.0 ** -9 * qs.cpu()[..., None]).all())
    ref = o.indexer_scores(qd, kd, w.cpu())
    fin = torch.isfinite(ref)
    assert torch.equal(torch.isfinite(out), fin)
    scale = ref[fin].abs().mean()
    assert bool(((out[fin] - ref[fin]).abs() <= 1e-4 * ref[fin].abs() + 1e-5 * scale).all())
