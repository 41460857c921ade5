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


def random_int8_linear(out_f: int, in_f: int, rng, scale_lo=1e-3, scale_hi=1e-1, std=0.02):
    """A pre-quantised linear: per-output-channel scales log-uniform in
    [scale_lo, scale_hi] and int8 values ``clip(rint(W / s), -127, 127)`` of
    N(0, std) weights, so the effective weights ``s * q`` keep the scale of
    random-init BERT weights (coarse channels round to few levels)."""
    s = np.exp(rng.uniform(np.log(scale_lo), np.log(scale_hi), size=out_f)).astype(np.float32)
    w = rng.standard_normal((out_f, in_f)) * std
    q = np.clip(np.rint(w / s[:, None]), -127, 127).astype(np.int8)
    return q, s
