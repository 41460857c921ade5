"""Integer-exact oracle for the int8 weight/activation format (test oracle only).

The reference has no int8 matmul (its compute precisions are F32/F16/BF16,
``crates/jammi-numerics/src/precision.rs:36-51``), so this format is defined
by this project:

* weights  ``W [out, in]`` -> ``Wq int8`` with one symmetric scale per output
  channel: ``amax = max|W_row|``, ``s = amax / 127``,
  ``Wq = clamp(rint(W * (127 / amax)), -127, 127)`` (all f32 arithmetic,
  round-half-to-even; an all-zero row gets ``s = 0`` and ``Wq = 0``);
* activations ``x [tokens, K]`` -> per-token int8 with the same rule;
* ``acc = sum_k xq * Wq`` in int32 (exact: ``|acc| <= K * 127^2 < 2^31`` for
  ``K <= 133 000``);
* ``y = float(acc) * (s_x * s_w) + b``.

The activation quantiser is restated in float32 so that, given the same bf16
input, the device quantiser's int8 output and scale are bit-identical.
"""
from __future__ import annotations

import numpy as np

from .bert import BertConfig, weight_prefix, layer_norm, gelu_erf, extended_attention_mask, softmax_last
import math


def quantize_rows(x):
    """Per-row symmetric int8: returns ``(q int8 [R,K], scale f32 [R])``."""
    x = np.asarray(x, dtype=np.float32)
    amax = np.abs(x).max(axis=-1)
    safe = np.where(amax > 0, amax, np.float32(1.0)).astype(np.float32)
    inv = (np.float32(127.0) / safe).astype(np.float32)
    inv = np.where(amax > 0, inv, np.float32(0.0)).astype(np.float32)
    prod = (x * inv[..., None]).astype(np.float32)
    q = np.clip(np.rint(prod), -127, 127).astype(np.int8)
    scale = (amax / np.float32(127.0)).astype(np.float32)
    return q, scale


def gemm_s8_s32(aq, bq):
    """``acc[m, n] = sum_k aq[m, k] * bq[n, k]`` exactly, as int32."""
    acc = aq.astype(np.int64) @ bq.astype(np.int64).T
    assert np.abs(acc).max(initial=0) < 2**31
    return acc.astype(np.int32)


def dequant(acc, s_tok, s_ch, bias=None):
    y = acc.astype(np.float64) * (s_tok.astype(np.float64)[:, None] * s_ch.astype(np.float64)[None, :])
    return y if bias is None else y + bias


def quant_linear(x, wq, ws, b):
    """int8 ``Linear``: per-token quant of ``x``, integer GEMM, dequant + bias."""
    shp = x.shape
    x2 = x.reshape(-1, shp[-1])
    q, s = quantize_rows(x2.astype(np.float32))
    y = dequant(gemm_s8_s32(q, wq), s, ws, b)
    return y.reshape(*shp[:-1], wq.shape[0])


LINEARS = ("attention.self.query", "attention.self.key", "attention.self.value",
           "attention.output.dense", "intermediate.dense", "output.dense")


def quantize_bert_weights(weights: dict, cfg: BertConfig) -> dict:
    """Per-output-channel int8 copies of the six per-layer linears:
    ``<name>.weight_q`` (int8) and ``<name>.weight_scale`` (f32)."""
    p = weight_prefix(weights)
    out = {}
    for n in range(cfg.num_hidden_layers):
        for lin in LINEARS:
            k = f"{p}encoder.layer.{n}.{lin}"
            if k + ".weight_q" in weights:
                out[k + ".weight_q"] = np.asarray(weights[k + ".weight_q"], dtype=np.int8)
                out[k + ".weight_scale"] = np.asarray(weights[k + ".weight_scale"], dtype=np.float32)
            else:
                q, s = quantize_rows(np.asarray(weights[k + ".weight"], dtype=np.float32))
                out[k + ".weight_q"] = q
                out[k + ".weight_scale"] = s
    return out


def bert_int8_forward_hidden(weights: dict, cfg: BertConfig, input_ids, mask):
    """BERT forward with the six linears in the int8 format above; embeddings,
    attention, LayerNorm and GELU in float64 (the same structure as
    ``oracle.bert.bert_forward_hidden``)."""
    ids = np.asarray(input_ids, dtype=np.int64)
    B, S = ids.shape
    p = weight_prefix(weights)
    qw = quantize_bert_weights(weights, cfg)
    H, nh = cfg.hidden_size, cfg.num_attention_heads
    d = H // nh
    eps = cfg.layer_norm_eps
    g = lambda k: np.asarray(weights[p + k], dtype=np.float64)

    def lin(x, name):
        k = f"{p}{name}"
        return quant_linear(x, qw[k + ".weight_q"], qw[k + ".weight_scale"], g(name + ".bias"))

    x = g("embeddings.word_embeddings.weight")[ids]
    x = x + g("embeddings.token_type_embeddings.weight")[0]
    x = x + g("embeddings.position_embeddings.weight")[:S][None]
    x = layer_norm(x, g("embeddings.LayerNorm.weight"), g("embeddings.LayerNorm.bias"), eps)
    ext = extended_attention_mask(mask).astype(np.float64)
    for n in range(cfg.num_hidden_layers):
        pre = f"encoder.layer.{n}."
        q = lin(x, pre + "attention.self.query").reshape(B, S, nh, d).transpose(0, 2, 1, 3)
        k = lin(x, pre + "attention.self.key").reshape(B, S, nh, d).transpose(0, 2, 1, 3)
        v = lin(x, pre + "attention.self.value").reshape(B, S, nh, d).transpose(0, 2, 1, 3)
        probs = softmax_last((q @ k.transpose(0, 1, 3, 2)) / math.sqrt(d) + ext)
        ctx = (probs @ v).transpose(0, 2, 1, 3).reshape(B, S, H)
        a = lin(ctx, pre + "attention.output.dense")
        x1 = layer_norm(a + x, g(pre + "attention.output.LayerNorm.weight"),
                        g(pre + "attention.output.LayerNorm.bias"), eps)
        f = gelu_erf(lin(x1, pre + "intermediate.dense"))
        o = lin(f, pre + "output.dense")
        x = layer_norm(o + x1, g(pre + "output.LayerNorm.weight"), g(pre + "output.LayerNorm.bias"), eps)
    return x


# ── bf16 storage between the int8 GEMMs ─────────────────────────────────────
#
# The int8 format keeps every activation tensor between two operators in
# bf16, as the reference's own BF16 compute precision does: each candle op
# (``Linear``, ``gelu_erf``, ``layer_norm``, the attention matmuls) returns a
# bf16 tensor (crates/jammi-encoders/src/bert.rs:143-154,164-167,187-190,
# 199-202; crates/jammi-encoders/src/layer_norm.rs:55-65).  The per-token
# quantiser therefore sees bf16 values and picks its int8 codes from them.
# ``bert_int8_bf16_forward`` restates the int8 forward with those rounding
# points, so that its int8 codes are the ones the device picks; the float64
# ``bert_int8_forward_hidden`` above keeps unrounded activations and drifts
# from them by one code at rounding boundaries.

_F64_DROP = np.uint64(45)            # 52 - 7 mantissa bits dropped by bf16
_F64_HALF_M1 = np.uint64((1 << 44) - 1)
_F64_KEEP = ~np.uint64((1 << 45) - 1)


def bf16_round(x):
    """Round float64 values to the nearest bfloat16, ties to even (returned
    as float32, which holds every bf16 value exactly).

    Works on the float64 bit pattern: add just under half of the dropped
    range plus the kept LSB (the ties-to-even rule), then clear the dropped
    bits.  Exact for every value in bf16's normal range."""
    x = np.ascontiguousarray(np.asarray(x, dtype=np.float64))
    u = x.view(np.uint64)
    u = (u + _F64_HALF_M1 + ((u >> _F64_DROP) & np.uint64(1))) & _F64_KEEP
    return u.view(np.float64).astype(np.float32)


def bf16_round_f32(x):
    """float32 values stored as bf16 (round to nearest, ties to even) -- the
    rounding a float32 result takes when the device stores it as bf16.
    Returned as float32."""
    u = np.ascontiguousarray(np.asarray(x, dtype=np.float32)).view(np.uint32)
    u = (u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))) & np.uint32(0xFFFF0000)
    return u.view(np.float32)


def gemm_s8_exact(aq, bq):
    """``acc[m, n] = sum_k aq[m, k] * bq[n, k]`` exactly, on float32 BLAS: K is
    cut into chunks of 1024, whose partial sums are integers of magnitude
    <= 1024 * 128 * 128 = 2^24, every one exactly representable in float32
    whatever order the BLAS adds them in; the chunks are summed in float64
    (exact below 2^53).  Returns float64 holding the integers."""
    a = np.asarray(aq, dtype=np.float32)
    b = np.asarray(bq, dtype=np.float32)
    K = a.shape[1]
    if K <= 1024:
        return (a @ b.T).astype(np.float64)
    acc = np.zeros((a.shape[0], b.shape[0]), dtype=np.float64)
    for k0 in range(0, K, 1024):
        acc += a[:, k0:k0 + 1024] @ b[:, k0:k0 + 1024].T
    return acc


def dequant_f32(acc, s_tok, s_ch, bias, resid=None):
    """The dequantising epilogue in the device's float32 operation order:
    ``s = f32(s_tok * s_ch)``, ``y = fma(f32(acc), s, bias)`` (one rounding:
    the product of two float32 values is exact in float64), then
    ``y + resid`` in float32.  Returns float32."""
    a = np.asarray(acc, dtype=np.float32)                             # int -> f32 rounding
    s = np.multiply.outer(np.asarray(s_tok, np.float32), np.asarray(s_ch, np.float32))
    bias = np.asarray(bias, np.float32)
    if bias.any():
        y = a.astype(np.float64) * s
        y += bias.astype(np.float64)[None, :]
        y = y.astype(np.float32)
    else:  # fma(a, s, 0) is the float32 product, rounded once
        y = a * s
    if resid is not None:
        y += np.asarray(resid, np.float32)
    return y


_POOL = None


def _row_blocks(fn, rows, block):
    """Runs ``fn(r0, r1)`` over row blocks on a thread pool (numpy's ufunc
    loops and BLAS release the GIL, so the blocks run in parallel)."""
    global _POOL
    import concurrent.futures as cf
    import os
    if _POOL is None:
        _POOL = cf.ThreadPoolExecutor(max_workers=max(1, min(16, os.cpu_count() or 1)))
    futs = [_POOL.submit(fn, r0, min(rows, r0 + block)) for r0 in range(0, rows, block)]
    for f in futs:
        f.result()


def int8_linear_bf16(x, wq, ws, bias, resid=None, block=512):
    """One int8 linear of the bf16-storage forward: per-token quantisation of
    the bf16 input ``x`` (``quantize_rows``), the exact integer product,
    ``dequant_f32`` (+ the residual), stored as bf16.  float32 in and out."""
    x = np.asarray(x, dtype=np.float32)
    T = x.shape[0]
    wf = np.asarray(wq, dtype=np.float32)
    out = np.empty((T, wf.shape[0]), dtype=np.float32)

    def run(r0, r1):
        q, s = quantize_rows(x[r0:r1])
        y = dequant_f32(gemm_s8_exact(q, wf), s, ws, bias,
                        None if resid is None else resid[r0:r1])
        out[r0:r1] = bf16_round_f32(y)

    _row_blocks(run, T, block)
    return out


LOG2E = 1.4426950408889634

# The attention kernels' block structure: keys in blocks of `block`, p taken
# against a reference maximum raised only when a block's maximum exceeds it
# by more than `threshold` (log2 units).  The tcgen05 kernel (the default)
# uses 128 / 8; the mma.sync kernel 64 / 0 (every rise rescales).
ATTN_TC = (128, 8.0)
ATTN_MMA = (64, 0.0)


def attention_bf16_p(q, k, v, scale, block=128, threshold=8.0):
    """softmax(q k^T * scale) v for one row and head, with P stored as bf16 as
    the device's P V product takes it: per key block, p = 2^(s * scale *
    log2(e) - m) against the reference maximum m (the first block's maximum,
    raised -- with O and the sum rescaled -- only when a later block's exceeds
    it by more than `threshold`); O accumulates bf16(p) V, the sum the
    unrounded p; the result is O / sum.  float64 otherwise."""
    t = (np.asarray(q, np.float64) @ np.asarray(k, np.float64).T) * (scale * LOG2E)
    v = np.asarray(v, np.float64)
    rows, n = t.shape
    mref = np.full(rows, -np.inf)
    lsum = np.zeros(rows)
    o = np.zeros((rows, v.shape[1]))
    for b0 in range(0, n, block):
        tb = t[:, b0:b0 + block]
        mb = tb.max(axis=1)
        first = np.isneginf(mref)
        up = ~first & (mb > mref + threshold)
        if up.any():
            alpha = np.exp2(mref[up] - mb[up])
            o[up] *= alpha[:, None]
            lsum[up] *= alpha
            mref[up] = mb[up]
        mref[first] = mb[first]
        p = np.exp2(tb - mref[:, None])
        lsum += p.sum(axis=1)
        o += bf16_round(p).astype(np.float64) @ v[b0:b0 + block]
    return o / lsum[:, None]


def _row_offsets(lens):
    lens = np.asarray(lens, dtype=np.int64)
    cu = np.zeros(len(lens) + 1, dtype=np.int64)
    np.cumsum(lens, out=cu[1:])
    return cu


def bert_int8_bf16_forward(weights: dict, cfg: BertConfig, input_ids, lens, attention=ATTN_TC):
    """The int8 BERT forward with bf16 storage between operators, over the
    valid tokens of each row only (padding never reaches a valid row: the
    -10000 mask of crates/jammi-encoders/src/mask.rs:14-20 underflows to 0).

    Layer structure as ``Bert::forward_hidden`` (bert.rs:257-276):
    embeddings word + type[0] + position summed in f32 from bf16 tables, LN,
    bf16 (bert.rs:102-111); per layer the Q, K, V int8 linears -> bf16;
    softmax(QK^T / sqrt(d)) V per row and head with P stored as bf16 in the
    block structure of the attention kernel (``attention_bf16_p``; ``attention``
    = (block, threshold), ``ATTN_TC`` or ``ATTN_MMA``) -> bf16 context;
    attention-out int8 linear + residual -> bf16, LN -> bf16
    (bert.rs:164-167); FFN1 int8 linear -> bf16, exact-erf GELU -> bf16
    (bert.rs:187-190); FFN2 int8 linear + residual -> bf16, LN -> bf16
    (bert.rs:199-202).  LayerNorm, the rest of attention and GELU are
    evaluated in float64 and rounded once to bf16.

    Returns ``(hidden [T, H] float32 of bf16 values, cu [B+1])`` with the
    rows packed: row b is ``hidden[cu[b]:cu[b+1]]``."""
    ids = np.asarray(input_ids, dtype=np.int64)
    lens = np.asarray(lens, dtype=np.int64)
    B = ids.shape[0]
    if lens.max(initial=0) > cfg.max_position_embeddings:
        raise ValueError("row longer than max_position_embeddings")
    p = weight_prefix(weights)
    qw = quantize_bert_weights(weights, cfg)
    H, nh = cfg.hidden_size, cfg.num_attention_heads
    d = H // nh
    eps = cfg.layer_norm_eps
    f32 = lambda k: np.asarray(weights[p + k], dtype=np.float32)
    cu = _row_offsets(lens)
    T = int(cu[-1])
    tok = np.concatenate([ids[b, :lens[b]] for b in range(B)]) if T else np.zeros(0, np.int64)
    pos = np.concatenate([np.arange(n) for n in lens]) if T else np.zeros(0, np.int64)

    def ln(x, name):
        g = f32(name + ".weight").astype(np.float64)
        bb = f32(name + ".bias").astype(np.float64)
        out = np.empty(x.shape, dtype=np.float32)

        def run(r0, r1):
            out[r0:r1] = bf16_round(layer_norm(x[r0:r1].astype(np.float64), g, bb, eps))

        _row_blocks(run, x.shape[0], 512)
        return out

    def lin(x, name, resid=None):
        k = f"{p}{name}"
        return int8_linear_bf16(x, qw[k + ".weight_q"], qw[k + ".weight_scale"], f32(name + ".bias"), resid)

    # BertEmbeddings (bert.rs:102-111): (word + type[0]) + position in f32
    # from the bf16 tables
    e = bf16_round_f32(f32("embeddings.word_embeddings.weight")[tok])
    e += bf16_round_f32(f32("embeddings.token_type_embeddings.weight")[0])[None, :]
    e += bf16_round_f32(f32("embeddings.position_embeddings.weight"))[pos]
    x = ln(e, "embeddings.LayerNorm")
    scale = 1.0 / math.sqrt(d)
    for n in range(cfg.num_hidden_layers):
        pre = f"encoder.layer.{n}."
        qkv = np.concatenate([lin(x, pre + "attention.self." + nm) for nm in ("query", "key", "value")],
                             axis=1)
        ctx = np.empty((T, H), dtype=np.float32)

        def attend(b0, b1):
            for b in range(b0, b1):
                r0, r1 = int(cu[b]), int(cu[b + 1])
                if r1 == r0:
                    continue
                m = r1 - r0
                blk = qkv[r0:r1].astype(np.float64)
                for hh in range(nh):
                    c0 = hh * d
                    ctx[r0:r1, c0:c0 + d] = bf16_round(attention_bf16_p(
                        blk[:, c0:c0 + d], blk[:, H + c0:H + c0 + d], blk[:, 2 * H + c0:2 * H + c0 + d],
                        scale, *attention))

        _row_blocks(attend, B, 4)
        a = lin(ctx, pre + "attention.output.dense", resid=x)
        x1 = ln(a, pre + "attention.output.LayerNorm")
        h = lin(x1, pre + "intermediate.dense")
        g = np.empty(h.shape, dtype=np.float32)

        def act(r0, r1):
            g[r0:r1] = bf16_round(gelu_erf(h[r0:r1].astype(np.float64)))

        _row_blocks(act, T, 256)
        o = lin(g, pre + "output.dense", resid=x1)
        x = ln(o, pre + "output.LayerNorm")
    return x, cu


def pool_packed(hidden, cu, strategy=0):
    """Mean (strategy 0) or CLS (1) pooling of packed rows, then the L2 norm of
    ``pool_and_normalize`` (crates/jammi-encoders/src/pooling.rs:31-66,
    123-148); an empty row pools to the zero vector."""
    from .bert import l2_normalize
    B = len(cu) - 1
    out = np.zeros((B, hidden.shape[1]), dtype=np.float64)
    for b in range(B):
        r0, r1 = int(cu[b]), int(cu[b + 1])
        if r1 > r0:
            out[b] = hidden[r0:r1].astype(np.float64).mean(axis=0) if strategy == 0 else hidden[r0]
    return l2_normalize(out)


def bert_int8_bf16_embed(weights: dict, cfg: BertConfig, input_ids, lens, strategy=0,
                         attention=ATTN_TC):
    """``Bert::forward`` (bert.rs:279-282) of the int8 format with bf16 storage:
    pooled, L2-normalised ``[B, H]``."""
    h, cu = bert_int8_bf16_forward(weights, cfg, input_ids, lens, attention)
    return pool_packed(h, cu, strategy)


def random_int8_linear(out_f: int, in_f: int, rng, scale_lo=1e-3, scale_hi=1e-1, std=0.02):
    """A pre-quantised linear: per-output-channel scales log-uniform in
    [scale_lo, scale_hi] and int8 values ``clip(rint(W / s), -127, 127)`` of
    N(0, std) weights, so the effective weights ``s * q`` keep the scale of
    random-init BERT weights (coarse channels round to few levels)."""
    s = np.exp(rng.uniform(np.log(scale_lo), np.log(scale_hi), size=out_f)).astype(np.float32)
    w = rng.standard_normal((out_f, in_f)) * std
    q = np.clip(np.rint(w / s[:, None]), -127, 127).astype(np.int8)
    return q, s
