"""ctypes binding of libdsa_b200.so (the C ABI in include/dsa_b200.h).

The library is loaded from this directory.  There is no fallback: if it is
missing or a call fails, an exception is raised.  Tensors passed in must be
CUDA tensors on the current device, 16-byte aligned; the plain entry points
take them contiguous, the ``*_ex`` ones with any strides whose innermost
dimension is contiguous (see :class:`Layout`).  The wrappers in
lightning_indexer.py / dsa_attention.py make sure of that.  Every call is
enqueued on torch's current CUDA stream.
"""
from __future__ import annotations

import ctypes
import os

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
# DSA_LIB_VARIANT=checked loads the checked build (libdsa_b200_checked.so)
LIB_PATH = os.path.join(HERE, "libdsa_b200_checked.so" if os.environ.get("DSA_LIB_VARIANT") == "checked"
                        else "libdsa_b200.so")

DSA_OK, DSA_ERR_INVALID, DSA_ERR_UNSUPPORTED, DSA_ERR_CUDA, DSA_ERR_TIMEOUT = 0, -1, -2, -3, -4
DSA_F32, DSA_BF16, DSA_F16, DSA_FP8_E4M3 = 0, 1, 2, 3
_DTYPES = {torch.float32: DSA_F32, torch.bfloat16: DSA_BF16, torch.float16: DSA_F16,
           torch.float8_e4m3fn: DSA_FP8_E4M3}

_lib = None


class Layout(ctypes.Structure):
    """struct dsa_layout: element strides (outermost first) of q_idx [B,T_q,HI,DI],
    k_idx [B,T_k,DI], w_idx [B,T_q,HI], Q/K/V [B,T,H,D], and the per-batch step
    of the first query row (row blocks of one sequence in one call)."""
    _fields_ = [("q", ctypes.c_int64 * 3), ("k", ctypes.c_int64 * 2), ("w", ctypes.c_int64 * 2),
                ("Q", ctypes.c_int64 * 3), ("K", ctypes.c_int64 * 3), ("V", ctypes.c_int64 * 3),
                ("row_bstep", ctypes.c_int64)]


def layout(q=None, k=None, w=None, Q=None, K=None, V=None, row_bstep=0) -> Layout:
    """A Layout from the given tensors' strides (unlisted tensors: zeros, unused by the callee)."""
    L = Layout()
    for name, t, n in (("q", q, 3), ("k", k, 2), ("w", w, 2), ("Q", Q, 3), ("K", K, 3), ("V", V, 3)):
        if t is not None:
            getattr(L, name)[:] = list(t.stride()[:n])
    L.row_bstep = int(row_bstep)
    return L


def lib() -> ctypes.CDLL:
    """The loaded library (loaded on first use)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"{LIB_PATH} is not built; run `python dsa-cpu-topk_b200/build.py` "
                "(or __graft_entry__.build()) first")
        L = ctypes.CDLL(LIB_PATH)
        p, i64, i32, f32, sz = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_float, ctypes.c_size_t
        L.dsa_version.restype = i32
        L.dsa_last_error_string.restype = ctypes.c_char_p
        L.dsa_indexer_scores.argtypes = [p, p, p, p, i64, i64, i64, i64, i64, i64, i32, i32, p]
        L.dsa_topk_select.argtypes = [p, i64, i64, i64, i64, i64, i32, i64, p, p, p, i64, p]
        L.dsa_sparse_attn_threshold.argtypes = [p, p, p, p, p, p, i64, i64, i64, i64, i64, i64, i64,
                                                f32, i32, p]
        L.dsa_sparse_attn.argtypes = [p, p, i64, p, p, p, p, p, p, i64, i64, i64, i64, i64, i64, i64,
                                      f32, i32, p]
        L.dsa_bitmap_words.argtypes = [i64]
        L.dsa_bitmap_words.restype = i64
        L.dsa_kept_bitmap.argtypes = [p, p, p, i64, i64, i64, i64, i64, p]
        L.dsa_topk_select_bitmap.argtypes = [p, i64, i64, i64, i64, i32, i64, p, p, p, i64, p]
        L.dsa_sparse_attn_bitmap.argtypes = [p, i64, p, p, p, p, i64, i64, i64, i64, i64, i64, i64,
                                             f32, i32, p]
        L.dsa_topk_select_bitmap_workspace_bytes.argtypes = [i64, i64]
        L.dsa_topk_select_bitmap_workspace_bytes.restype = sz
        L.dsa_topk_select_bitmap_ws.argtypes = [p, i64, i64, i64, i64, i64, i32, i64, p, p, p, i64, p, sz, p]
        L.dsa_device_status.argtypes = [p]
        L.dsa_device_status.restype = i32
        L.dsa_forward_workspace_bytes.argtypes = [i64, i64, i64, i64]
        L.dsa_forward_workspace_bytes.restype = sz
        L.dsa_forward.argtypes = [p, p, p, p, p, p, p, i64, i64, i64, i64, i64, i64, i64, i64, i64, i64,
                                  i32, i32, p, sz, p]
        lp = ctypes.POINTER(Layout)
        L.dsa_layout_contiguous.argtypes = [lp, i64, i64, i64, i64, i64, i64, i64]
        L.dsa_layout_contiguous.restype = None
        L.dsa_indexer_scores_ex.argtypes = [p, p, p, p, i64, i64, i64, i64, i64, i64, i32, i32, lp, p]
        L.dsa_topk_select_ex.argtypes = [p, i64, i64, i64, i64, i64, i64, i32, i64, p, p, p, i64, p, i64, p]
        L.dsa_sparse_attn_ex.argtypes = [p, p, i64, p, p, p, p, p, p, i64, i64, i64, i64, i64, i64, i64,
                                         f32, i32, lp, p]
        L.dsa_sparse_attn_bitmap_ex.argtypes = [p, i64, p, p, p, p, i64, i64, i64, i64, i64, i64, i64,
                                                f32, i32, lp, p, sz, p]
        L.dsa_sparse_attn_bitmap_workspace_bytes.argtypes = [i64, i64, i64, i64, i64, i32]
        L.dsa_sparse_attn_bitmap_workspace_bytes.restype = sz
        L.dsa_forward_workspace_bytes_ex.argtypes = [i64, i64, i64, i64, i64, i64, i32]
        L.dsa_forward_workspace_bytes_ex.restype = sz
        L.dsa_forward_ex.argtypes = [p, p, p, p, p, p, p, i64, i64, i64, i64, i64, i64, i64, i64, i64, i64,
                                     i32, i32, lp, p, sz, p]
        L.dsa_quantize_fp8_rows.argtypes = [p, i32, i64, i64, i64, p, p, p]
        L.dsa_indexer_scores_fp8.argtypes = [p, p, p, p, p, i64, i64, i64, i64, i64, i64, i32, lp, p]
        L.dsa_debug_checks_enabled.restype = i32
        L.dsa_debug_status.argtypes = [p]
        L.dsa_debug_status.restype = i32
        L.dsa_forward_noalloc.argtypes = [p, p, p, p, p, p, p, i64, i64, i64, i64, i64, i64, i64, i64, i64,
                                          i64, i32, i32, p]
        for name in ("dsa_indexer_scores", "dsa_topk_select", "dsa_sparse_attn_threshold",
                     "dsa_sparse_attn", "dsa_forward", "dsa_kept_bitmap", "dsa_sparse_attn_bitmap",
                     "dsa_topk_select_bitmap", "dsa_indexer_scores_ex", "dsa_topk_select_ex",
                     "dsa_sparse_attn_ex", "dsa_sparse_attn_bitmap_ex", "dsa_forward_ex",
                     "dsa_forward_noalloc", "dsa_quantize_fp8_rows", "dsa_indexer_scores_fp8",
                     "dsa_topk_select_bitmap_ws"):
            getattr(L, name).restype = i32
        _lib = L
    return _lib


def _check(rc: int, what: str) -> None:
    if rc == DSA_OK:
        return
    msg = f"{what}: {lib().dsa_last_error_string().decode(errors='replace')}"
    if rc == DSA_ERR_INVALID:
        raise AssertionError(msg)
    raise RuntimeError(msg)


def dtype_code(t: torch.Tensor) -> int:
    try:
        return _DTYPES[t.dtype]
    except KeyError:
        raise AssertionError(f"unsupported dtype {t.dtype} (fp32, bf16, fp16; e4m3 for indexer inputs)") from None


def prep(t: torch.Tensor) -> torch.Tensor:
    """Contiguous, 16-byte-aligned CUDA tensor (copies only when needed)."""
    assert t.is_cuda, "inputs must be CUDA tensors"
    t = t.contiguous()
    if t.data_ptr() % 16:
        t = t.clone()
    return t


def prep_strided(t: torch.Tensor) -> torch.Tensor:
    """A CUDA tensor the ``*_ex`` entry points take as it is: innermost dimension
    contiguous, every other stride a multiple of 16 bytes, 16-byte-aligned base
    (copies only when one of those fails)."""
    assert t.is_cuda, "inputs must be CUDA tensors"
    e = t.element_size()
    ok = (t.stride(-1) == 1 or t.shape[-1] == 1) and t.data_ptr() % 16 == 0 and \
        all((st * e) % 16 == 0 for st, n in zip(t.stride()[:-1], t.shape[:-1]) if n > 1)
    if ok:
        return t
    t = t.contiguous()
    if t.data_ptr() % 16:
        t = t.clone()
    return t


def _ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def indexer_scores(q, k, w, scores, *, q_row0=0, fill_upper=True):
    B, T_q, HI, DI = q.shape
    T_k = k.shape[1]
    _check(lib().dsa_indexer_scores(_ptr(q), _ptr(k), _ptr(w), _ptr(scores), B, T_q, T_k, q_row0,
                                    HI, DI, dtype_code(q), int(bool(fill_upper)), _stream()),
           "dsa_indexer_scores")


def topk_select(scores, n_rows, row_len, row_stride, k, thr, idx=None, cnt=None, idx_cap=0, *,
                causal=False, rows_per_batch=1, q_row0=0):
    _check(lib().dsa_topk_select(_ptr(scores), n_rows, row_len, row_stride, rows_per_batch, q_row0,
                                 int(bool(causal)), k, _ptr(thr), _ptr(idx), _ptr(cnt), idx_cap,
                                 _stream()), "dsa_topk_select")


def sparse_attn_threshold(scores, thr, Q, K, V, O, *, q_row0=0, scale=None):
    B, T_q, HQ, DQ = Q.shape
    T_k, DV = K.shape[1], V.shape[-1]
    scale = DQ ** -0.5 if scale is None else scale
    _check(lib().dsa_sparse_attn_threshold(_ptr(scores), _ptr(thr), _ptr(Q), _ptr(K), _ptr(V),
                                           _ptr(O), B, T_q, T_k, q_row0, HQ, DQ, DV, scale,
                                           dtype_code(Q), _stream()), "dsa_sparse_attn_threshold")


def sparse_attn(idx, cnt, idx_cap, scores, thr, Q, K, V, O, *, q_row0=0, scale=None):
    B, T_q, HQ, DQ = Q.shape
    T_k, DV = K.shape[1], V.shape[-1]
    scale = DQ ** -0.5 if scale is None else scale
    _check(lib().dsa_sparse_attn(_ptr(idx), _ptr(cnt), idx_cap, _ptr(scores), _ptr(thr), _ptr(Q),
                                 _ptr(K), _ptr(V), _ptr(O), B, T_q, T_k, q_row0, HQ, DQ, DV, scale,
                                 dtype_code(Q), _stream()), "dsa_sparse_attn")


def bitmap_words(T_k) -> int:
    return int(lib().dsa_bitmap_words(T_k))


def attn_tc_supported(Q, V) -> bool:
    """Whether dsa_sparse_attn_bitmap runs this dtype / head size (bf16 or fp16, DQ == DV in {64, 128})."""
    return (Q.dtype in (torch.bfloat16, torch.float16) and Q.shape[-1] == V.shape[-1]
            and Q.shape[-1] in (64, 128))


def kept_bitmap(scores, thr, bits, *, q_row0=0):
    B, T_q, T_k = scores.shape
    _check(lib().dsa_kept_bitmap(_ptr(scores), _ptr(thr), _ptr(bits), B, T_q, T_k, q_row0,
                                 bits.shape[-1], _stream()), "dsa_kept_bitmap")


def topk_select_bitmap_workspace_bytes(n_rows, words):
    return int(lib().dsa_topk_select_bitmap_workspace_bytes(n_rows, words))


def topk_select_bitmap(scores, k, thr, bits, cnt=None, *, causal=True, q_row0=0, row_bstep=0,
                       workspace=None):
    """Threshold (+ count) and kept-set bitmap of every row of scores [B, T_q, T_k].

    With a workspace (uint8 CUDA tensor of topk_select_bitmap_workspace_bytes)
    rows of 4K-32K entries take the sweep + resolve kernels."""
    B, T_q, T_k = scores.shape
    if workspace is None:
        assert row_bstep == 0, "row_bstep needs the workspace form"
        _check(lib().dsa_topk_select_bitmap(_ptr(scores), B * T_q, T_k, T_q, q_row0, int(bool(causal)), k,
                                            _ptr(thr), _ptr(cnt), _ptr(bits), bits.shape[-1], _stream()),
               "dsa_topk_select_bitmap")
        return
    _check(lib().dsa_topk_select_bitmap_ws(_ptr(scores), B * T_q, T_k, T_q, q_row0, row_bstep,
                                           int(bool(causal)), k,
                                           _ptr(thr), _ptr(cnt), _ptr(bits), bits.shape[-1], _ptr(workspace),
                                           workspace.numel(), _stream()),
           "dsa_topk_select_bitmap_ws")


def sparse_attn_bitmap(bits, Q, K, V, O, *, q_row0=0, scale=None):
    B, T_q, HQ, DQ = Q.shape
    T_k, DV = K.shape[1], V.shape[-1]
    scale = DQ ** -0.5 if scale is None else scale
    _check(lib().dsa_sparse_attn_bitmap(_ptr(bits), bits.shape[-1], _ptr(Q), _ptr(K), _ptr(V),
                                        _ptr(O), B, T_q, T_k, q_row0, HQ, DQ, DV, scale,
                                        dtype_code(Q), _stream()), "dsa_sparse_attn_bitmap")


def device_status() -> int:
    """Synchronise the current stream; DSA_OK or DSA_ERR_TIMEOUT (flag read and cleared)."""
    return int(lib().dsa_device_status(_stream()))


def forward_workspace_bytes(B, T_q, T_k, top_k, HQ=None, DV=None, qkv_dtype=None) -> int:
    """dsa_forward's workspace; with the head shape and Q/K/V dtype given, the
    _ex size that also holds the fp16 copy of V (bf16 inputs)."""
    if HQ is None:
        return int(lib().dsa_forward_workspace_bytes(B, T_q, T_k, top_k))
    return int(lib().dsa_forward_workspace_bytes_ex(B, T_q, T_k, top_k, HQ, DV, qkv_dtype))


def forward(q_idx, k_idx, w_idx, Q, K, V, O, top_k, workspace, *, q_row0=0):
    B, T_q, HI, DI = q_idx.shape
    T_k = k_idx.shape[1]
    HQ, DQ, DV = Q.shape[2], Q.shape[3], V.shape[3]
    _check(lib().dsa_forward(_ptr(q_idx), _ptr(k_idx), _ptr(w_idx), _ptr(Q), _ptr(K), _ptr(V),
                             _ptr(O), B, T_q, T_k, q_row0, HI, DI, HQ, DQ, DV, top_k,
                             dtype_code(q_idx), dtype_code(Q), _ptr(workspace),
                             workspace.numel() * workspace.element_size(), _stream()), "dsa_forward")


def forward_ex(q_idx, k_idx, w_idx, Q, K, V, O, top_k, workspace, *, q_row0=0, row_bstep=0):
    """dsa_forward_ex: strided inputs (key-side batch dimension may be a broadcast
    of size-1 / stride 0) and row blocks at q_row0 + b*row_bstep."""
    B, T_q, HI, DI = q_idx.shape
    T_k = k_idx.shape[1]
    HQ, DQ, DV = Q.shape[2], Q.shape[3], V.shape[3]
    L = layout(q_idx, k_idx, w_idx, Q, K, V, row_bstep)
    _check(lib().dsa_forward_ex(_ptr(q_idx), _ptr(k_idx), _ptr(w_idx), _ptr(Q), _ptr(K), _ptr(V),
                                _ptr(O), B, T_q, T_k, q_row0, HI, DI, HQ, DQ, DV, top_k,
                                dtype_code(q_idx), dtype_code(Q), ctypes.byref(L), _ptr(workspace),
                                workspace.numel() * workspace.element_size(), _stream()), "dsa_forward_ex")


def indexer_scores_ex(q, k, w, scores, *, q_row0=0, row_bstep=0, fill_upper=True):
    B, T_q, HI, DI = q.shape
    T_k = k.shape[1]
    L = layout(q=q, k=k, w=w, row_bstep=row_bstep)
    _check(lib().dsa_indexer_scores_ex(_ptr(q), _ptr(k), _ptr(w), _ptr(scores), B, T_q, T_k, q_row0,
                                       HI, DI, dtype_code(q), int(bool(fill_upper)), ctypes.byref(L),
                                       _stream()), "dsa_indexer_scores_ex")


def topk_select_ex(scores, n_rows, row_len, row_stride, k, thr, idx=None, cnt=None, idx_cap=0, bits=None,
                   *, causal=False, rows_per_batch=1, q_row0=0, row_bstep=0):
    words = 0 if bits is None else bits.shape[-1]
    _check(lib().dsa_topk_select_ex(_ptr(scores), n_rows, row_len, row_stride, rows_per_batch, q_row0,
                                    row_bstep, int(bool(causal)), k, _ptr(thr), _ptr(idx), _ptr(cnt),
                                    idx_cap, _ptr(bits), words, _stream()), "dsa_topk_select_ex")


def sparse_attn_bitmap_workspace_bytes(B, T_q, T_k, HQ, DV, dtype_c) -> int:
    return int(lib().dsa_sparse_attn_bitmap_workspace_bytes(B, T_q, T_k, HQ, DV, dtype_c))


def sparse_attn_bitmap_ex(bits, Q, K, V, O, *, q_row0=0, row_bstep=0, scale=None, workspace=None):
    """Tensor-core attention over the kept-set bitmap.  ``workspace`` (uint8, at least
    sparse_attn_bitmap_workspace_bytes) enables block skipping and, for bf16 inputs,
    fp16 softmax weights."""
    B, T_q, HQ, DQ = Q.shape
    T_k, DV = K.shape[1], V.shape[-1]
    scale = DQ ** -0.5 if scale is None else scale
    L = layout(Q=Q, K=K, V=V, row_bstep=row_bstep)
    ws_bytes = 0 if workspace is None else workspace.numel() * workspace.element_size()
    _check(lib().dsa_sparse_attn_bitmap_ex(_ptr(bits), bits.shape[-1], _ptr(Q), _ptr(K), _ptr(V),
                                           _ptr(O), B, T_q, T_k, q_row0, HQ, DQ, DV, scale,
                                           dtype_code(Q), ctypes.byref(L), _ptr(workspace), ws_bytes,
                                           _stream()),
           "dsa_sparse_attn_bitmap_ex")


def sparse_attn_ex(idx, cnt, idx_cap, scores, thr, Q, K, V, O, *, q_row0=0, row_bstep=0, scale=None):
    """List form (idx given) or threshold form (idx None) over strided Q/K/V."""
    B, T_q, HQ, DQ = Q.shape
    T_k, DV = K.shape[1], V.shape[-1]
    scale = DQ ** -0.5 if scale is None else scale
    L = layout(Q=Q, K=K, V=V, row_bstep=row_bstep)
    _check(lib().dsa_sparse_attn_ex(_ptr(idx), _ptr(cnt), idx_cap, _ptr(scores), _ptr(thr), _ptr(Q),
                                    _ptr(K), _ptr(V), _ptr(O), B, T_q, T_k, q_row0, HQ, DQ, DV, scale,
                                    dtype_code(Q), ctypes.byref(L), _stream()), "dsa_sparse_attn_ex")


def forward_noalloc(q_idx, k_idx, w_idx, Q, K, V, O, top_k, *, q_row0=0):
    """dsa_forward_noalloc: the whole forward with the library's own fixed scratch
    (no workspace argument, nothing allocated)."""
    B, T_q, HI, DI = q_idx.shape
    T_k = k_idx.shape[1]
    HQ, DQ, DV = Q.shape[2], Q.shape[3], V.shape[3]
    _check(lib().dsa_forward_noalloc(_ptr(q_idx), _ptr(k_idx), _ptr(w_idx), _ptr(Q), _ptr(K), _ptr(V),
                                     _ptr(O), B, T_q, T_k, q_row0, HI, DI, HQ, DQ, DV, top_k,
                                     dtype_code(q_idx), dtype_code(Q), _stream()), "dsa_forward_noalloc")


def quantize_fp8_rows(x, out, scale):
    """Rows of x's last dimension -> e4m3 ``out`` and per-row ``scale`` (max|x| / 448)."""
    D = x.shape[-1]
    rows = x.numel() // D if D else 0
    assert x.stride(-1) == 1 and (x.dim() == 1 or x.is_contiguous()), "rows must be contiguous"
    _check(lib().dsa_quantize_fp8_rows(_ptr(x), dtype_code(x), rows, D, D, _ptr(out), _ptr(scale), _stream()),
           "dsa_quantize_fp8_rows")


def indexer_scores_fp8(q8, k8, w, k_scale, scores, *, q_row0=0, row_bstep=0, fill_upper=True):
    B, T_q, HI, DI = q8.shape
    T_k = k8.shape[1]
    L = layout(q=q8, k=k8, w=w, row_bstep=row_bstep)
    _check(lib().dsa_indexer_scores_fp8(_ptr(q8), _ptr(k8), _ptr(w), _ptr(k_scale), _ptr(scores), B, T_q, T_k,
                                        q_row0, HI, DI, int(bool(fill_upper)), ctypes.byref(L), _stream()),
           "dsa_indexer_scores_fp8")


def debug_status() -> int:
    """Bits set by the checked build's failed index checks since the last call (0 normally)."""
    return int(lib().dsa_debug_status(_stream()))
