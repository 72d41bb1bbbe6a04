"""GPU: dsa_forward_noalloc, the forward for callers that cannot allocate.

Some callers cannot call cudaMalloc where they run the forward: a host
framework that owns every byte of GPU memory through its own pool, or a
plugin that is only handed its input and output buffers.  They cannot
provide dsa_forward's workspace, so dsa_forward_noalloc keeps that workspace
in a fixed 32 MiB array inside the library.

The test calls it through the C ABI and checks its output against
dsa_forward's (the caller-workspace entry point) on two calls in a row, so a
stale or shared scratch array would show up, and checks that a shape needing
more than 32 MiB is refused.  It creates all of its own inputs and passes
both alone in a fresh process and after the other tests.  This file is
named so that pytest collects it last.
"""
import ctypes

import pytest
import torch

import dsa_oracle as o

pytestmark = pytest.mark.gpu


def _bind():
    import _native
    lib = _native.lib()
    p, i64, i32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
    f = lib.dsa_forward_noalloc
    f.argtypes = [p, p, p, p, p, p, p] + [i64] * 10 + [i32, i32, p]
    f.restype = i32
    return lib, f, _native


def _call(f, native, args, O, top_k):
    q, k, w, Q, K, V = args
    B, T_q, HI, DI = q.shape
    T_k, HQ, DQ, DV = k.shape[1], Q.shape[2], Q.shape[3], V.shape[3]
    ptr = lambda t: ctypes.c_void_p(t.data_ptr())
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    return f(ptr(q), ptr(k), ptr(w), ptr(Q), ptr(K), ptr(V), ptr(O), B, T_q, T_k, 0, HI, DI, HQ,
             DQ, DV, top_k, native.dtype_code(q), native.dtype_code(Q), stream)


@pytest.mark.parametrize("B,T,HI,DI,HQ,D,k,dtype,tol", [
    (16, 512, 4, 32, 4, 32, 32, torch.float32, 5e-4),     # config c1 (fits in the 32 MiB)
    (1, 1024, 8, 128, 16, 128, 96, torch.bfloat16, 2e-2),
])
def test_noalloc_matches_dsa_forward_twice(cuda, B, T, HI, DI, HQ, D, k, dtype, tol):
    from dsa_attention import dsa_forward
    lib, f, native = _bind()
    for seed in (0, 100):  # two calls in a row, different data
        args = [x.to(cuda).contiguous() for x in o.make_inputs(B, T, HI, DI, HQ, D, D, dtype=dtype,
                                                               seed0=seed)]
        ref = dsa_forward(*args, k)
        O = torch.full((B, T, HQ, D), float("nan"), device=cuda, dtype=torch.float32)
        rc = _call(f, native, args, O, k)
        assert rc == 0, lib.dsa_last_error_string().decode()
        torch.cuda.synchronize()
        assert torch.isfinite(O).all()
        assert (O - ref).abs().max().item() <= tol


def test_noalloc_rejects_shapes_beyond_its_scratch(cuda):
    lib, f, native = _bind()
    args = [x.to(cuda) for x in o.make_inputs(1, 4096, 1, 16, 1, 16, 16)]
    O = torch.empty((1, 4096, 1, 16), device=cuda)
    rc = _call(f, native, args, O, 64)   # 4096 x 4096 fp32 scores alone are 64 MiB
    assert rc == native.DSA_ERR_INVALID
    assert b"32" in lib.dsa_last_error_string() or b"scratch" in lib.dsa_last_error_string()
