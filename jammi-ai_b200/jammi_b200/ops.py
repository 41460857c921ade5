"""Single-op entry points over torch CUDA tensors (device pointers only).

Each function calls one C-ABI op of libjammi_b200.so on the current torch
stream.  They exist for op-level parity tests and for callers that compose
their own forward; the encoder forward itself runs entirely inside the
library (``jb_encode_text`` / ``jb_encode_image``).
"""
from __future__ import annotations

import torch

from . import _lib as L
from ._lib import check, lib

_DT = {torch.float32: L.DT_F32, torch.bfloat16: L.DT_BF16, torch.float16: L.DT_F16, torch.int8: L.DT_S8,
       torch.int32: L.DT_S32}


def _s(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _p(t):
    return 0 if t is None else t.data_ptr()


def _contig(*ts):
    for t in ts:
        if t is not None and not t.is_contiguous():
            raise ValueError("tensors must be contiguous")


def sync(device=None):
    """``jb_op_sync``: synchronise the current stream and raise on a device-side timeout."""
    check(lib().jb_op_sync(torch.cuda.current_stream(device).cuda_stream))


def linear(a: torch.Tensor, w: torch.Tensor, bias=None, residual=None, epilogue: int = L.EPI_NONE,
           out_dtype=None) -> torch.Tensor:
    """``epi(a @ w.T + bias)``; a [M, K], w [N, K] both f32 or both bf16."""
    _contig(a, w, bias, residual)
    M, K = a.shape
    N = w.shape[0]
    out_dtype = out_dtype or a.dtype
    c = torch.empty((M, N), dtype=out_dtype, device=a.device)
    check(lib().jb_op_linear(_p(a), _DT[a.dtype], _p(w), _DT[w.dtype], _p(bias), _p(residual),
                             _p(c), _DT[out_dtype], M, N, K, epilogue, _s(a)))
    return c


def linear_s8(aq: torch.Tensor, a_scale, wq: torch.Tensor, w_scale, bias=None, residual=None,
              epilogue: int = L.EPI_NONE, out_dtype=torch.int32) -> torch.Tensor:
    """int8 linear: s32 accumulators (out_dtype int32) or dequantised output."""
    _contig(aq, a_scale, wq, w_scale, bias, residual)
    M, K = aq.shape
    N = wq.shape[0]
    c = torch.empty((M, N), dtype=out_dtype, device=aq.device)
    check(lib().jb_op_linear_s8(_p(aq), _p(a_scale), _p(wq), _p(w_scale), _p(bias), _p(residual),
                                _p(c), _DT[out_dtype], M, N, K, epilogue, _s(aq)))
    return c


def quantize_rows(x: torch.Tensor, activation: int = L.EPI_NONE):
    """Per-row int8 of x, or of activation(x) rounded to x's dtype
    (activation EPI_GELU): returns (q int8 [R, C], scale f32 [R])."""
    _contig(x)
    R, C = x.shape
    q = torch.empty((R, C), dtype=torch.int8, device=x.device)
    s = torch.empty((R,), dtype=torch.float32, device=x.device)
    if activation == L.EPI_NONE:
        check(lib().jb_op_quantize_rows(_p(x), _DT[x.dtype], _p(q), _p(s), R, C, _s(x)))
    else:
        check(lib().jb_op_quantize_rows_act(_p(x), _DT[x.dtype], int(activation), _p(q), _p(s), R, C,
                                            _s(x)))
    return q, s


def layernorm(x: torch.Tensor, gamma, beta, eps: float, residual=None) -> torch.Tensor:
    _contig(x, gamma, beta, residual)
    R, C = x.shape
    y = torch.empty_like(x)
    check(lib().jb_op_layernorm(_p(x), _p(residual), _p(gamma), _p(beta), _p(y), _DT[x.dtype], R, C,
                                float(eps), _s(x)))
    return y


def attention(qkv: torch.Tensor, cu_seqlens: torch.Tensor, heads: int, max_len: int,
              causal: bool = False, tma: bool = False) -> torch.Tensor:
    """qkv [T, 3*heads*d] packed rows, cu_seqlens int32 [B+1] -> ctx [T, heads*d]
    (``causal``: query i sees keys j <= i of its row; ``tma``: pass the row
    count, which selects the model forwards' TMA / tcgen05 kernels)."""
    _contig(qkv, cu_seqlens)
    T, three_h = qkv.shape
    H = three_h // 3
    ctx = torch.empty((T, H), dtype=qkv.dtype, device=qkv.device)
    if tma:
        check(lib().jb_op_attention_rows(_p(qkv), _p(cu_seqlens), _p(ctx), _DT[qkv.dtype],
                                         cu_seqlens.numel() - 1, heads, H // heads, max_len, T,
                                         1 if causal else 0, _s(qkv)))
        return ctx
    fn = lib().jb_op_attention_causal if causal else lib().jb_op_attention
    check(fn(_p(qkv), _p(cu_seqlens), _p(ctx), _DT[qkv.dtype], cu_seqlens.numel() - 1, heads,
             H // heads, max_len, _s(qkv)))
    return ctx


def pool_normalize(hidden: torch.Tensor, cu_seqlens: torch.Tensor, pooling: int = L.POOL_MEAN):
    _contig(hidden, cu_seqlens)
    T, H = hidden.shape
    B = cu_seqlens.numel() - 1
    out = torch.empty((B, H), dtype=torch.float32, device=hidden.device)
    check(lib().jb_op_pool_normalize(_p(hidden), _DT[hidden.dtype], _p(cu_seqlens), _p(out), B, H,
                                     pooling, _s(hidden)))
    return out


def preprocess_rgb8(images, target: int, mean, std, device="cuda") -> torch.Tensor:
    """RGB8 ``[h, w, 3]`` arrays -> f32 [B, 3, target, target] on the device
    (``jb_op_preprocess_rgb8``: white square pad, Catmull-Rom resize, normalise)."""
    from .encoders import pack_rgb8
    buf, offs, ws, hs = pack_rgb8(images)
    dev = torch.device(device)
    d_buf = torch.from_numpy(buf).to(dev)
    d_off = torch.from_numpy(offs).to(dev)
    d_w = torch.from_numpy(ws).to(dev)
    d_h = torch.from_numpy(hs).to(dev)
    m = torch.tensor(list(mean), dtype=torch.float32)
    s = torch.tensor(list(std), dtype=torch.float32)
    out = torch.empty((len(images), 3, target, target), dtype=torch.float32, device=dev)
    max_side = int(max(max(int(a), int(b)) for a, b in zip(ws, hs))) if len(images) else 1
    check(lib().jb_op_preprocess_rgb8(_p(d_buf), _p(d_off), _p(d_w), _p(d_h), len(images), max_side,
                                      target, m.data_ptr(), s.data_ptr(), _p(out), _s(out)))
    return out


def set_attention_tcgen05(on: bool):
    """``jb_set_attention_tcgen05``: every bf16 head-dim-64 row on the tcgen05
    attention kernel (process-wide; on by default), or off: the mma.sync kernel."""
    lib().jb_set_attention_tcgen05(1 if on else 0)


def wait_flag(flag: torch.Tensor, expect: int, limit_ms: int):
    """``jb_op_wait_flag``: a bounded device-side wait until flag[0] == expect;
    on expiry the next ``sync`` raises JbError (JB_ERR_TIMEOUT)."""
    if flag.dtype != torch.int32 or flag.numel() < 1:
        raise ValueError("flag must be an int32 tensor")
    check(lib().jb_op_wait_flag(_p(flag), int(expect), int(limit_ms), _s(flag)))


THRESHOLD_KINDS = {"mean": 0, "median": 1}


def fit_binary_threshold(vectors: torch.Tensor, kind: str = "median") -> torch.Tensor:
    """Per-dimension threshold tau of a Binary sidecar over the first
    min(rows, 100000) rows of f32 ``vectors`` [rows, dim] ("mean" or "median")."""
    _contig(vectors)
    rows, dim = vectors.shape
    tau = torch.empty(dim, dtype=torch.float32, device=vectors.device)
    check(lib().jb_op_fit_binary_threshold(_p(vectors), rows, dim, THRESHOLD_KINDS[kind], _p(tau), _s(vectors)))
    return tau


def pack_threshold_bits(vectors: torch.Tensor, tau: torch.Tensor) -> torch.Tensor:
    """uint8 [rows, ceil(dim / 8)]: bit i = vectors[:, i] > tau[i], LSB-first."""
    _contig(vectors, tau)
    rows, dim = vectors.shape
    out = torch.empty((rows, (dim + 7) // 8), dtype=torch.uint8, device=vectors.device)
    check(lib().jb_op_pack_threshold_bits(_p(vectors), rows, dim, _p(tau), _p(out), _s(vectors)))
    return out


def exact_search(corpus: torch.Tensor, queries: torch.Tensor, k: int, tie_rank=None):
    """Exact cosine search: (idx int64 [q, min(k, n)], dist f32 [q, min(k, n)])
    in ascending (distance, tie rank) order; ``tie_rank`` int32/uint32 [n]
    (distinct) or None for row order.  Synchronises to surface input errors."""
    _contig(corpus, queries, tie_rank)
    n, dim = corpus.shape
    nq = queries.shape[0]
    scratch = torch.empty((nq, n), dtype=torch.float32, device=corpus.device)
    idx = torch.empty((nq, k), dtype=torch.int64, device=corpus.device)
    dist = torch.empty((nq, k), dtype=torch.float32, device=corpus.device)
    check(lib().jb_op_exact_search(_p(corpus), n, dim, _p(tie_rank), _p(queries), nq, k, _p(scratch),
                                   _p(idx), _p(dist), _s(corpus)))
    sync(corpus.device)
    kk = min(k, n)
    return idx[:, :kk], dist[:, :kk]
