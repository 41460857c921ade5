"""numpy restatement of the reference BERT encoder forward (test oracle only).

Follows, step for step:

* ``BertEmbeddings::forward``      crates/jammi-encoders/src/bert.rs:102-111
* ``BertSelfAttention::forward``   bert.rs:135-155 (scores / sqrt(d), additive
  mask, softmax over the last dim, P.V)
* ``BertSelfOutput`` / ``BertOutput``  bert.rs:164-167, 199-202 (LN(dense(x)+res))
* ``BertIntermediate``             bert.rs:187-190 (exact-erf GELU)
* ``BertLayer`` / layer loop       bert.rs:212-216, 272-274
* ``Bert::forward_hidden``         bert.rs:257-276 (SequenceTooLong, zero
  token types)
* ``extended_attention_mask``      crates/jammi-encoders/src/mask.rs:14-20
* ``LayerNorm::forward``           crates/jammi-encoders/src/layer_norm.rs:55-84
* ``pool_and_normalize``           crates/jammi-encoders/src/pooling.rs:31-148
* ``Linear``                       crates/jammi-lora/src/wrapper.rs:29-42
  (``y = x W^T + b`` with W stored [out, in])

Computation runs on the padded ``[B, S]`` layout with the reference's additive
``-10000`` mask, exactly as the reference does, in float64 by default (the
accuracy oracle) or float32.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np

try:  # scipy's erf is vectorised; math.erf is the fallback.
    from scipy.special import erf as _erf
except Exception:  # pragma: no cover
    _erf = np.vectorize(math.erf)

POOL_MEAN, POOL_CLS, POOL_MAX, POOL_WEIGHTED_MEAN = 0, 1, 2, 3
POOLING_NAMES = {"mean": POOL_MEAN, "cls": POOL_CLS, "max": POOL_MAX,
                 "weighted_mean": POOL_WEIGHTED_MEAN}


class SequenceTooLong(ValueError):
    """Mirror of ``EncoderError::SequenceTooLong`` (bert.rs:263-268)."""


@dataclass
class BertConfig:
    """``BertConfig`` (bert.rs:35-58): HF ``config.json`` fields."""
    hidden_size: int
    num_hidden_layers: int
    num_attention_heads: int
    intermediate_size: int
    vocab_size: int
    max_position_embeddings: int
    type_vocab_size: int = 2
    layer_norm_eps: float = 1e-12

    @classmethod
    def from_dict(cls, d: dict) -> "BertConfig":
        return cls(
            hidden_size=int(d["hidden_size"]),
            num_hidden_layers=int(d["num_hidden_layers"]),
            num_attention_heads=int(d["num_attention_heads"]),
            intermediate_size=int(d["intermediate_size"]),
            vocab_size=int(d["vocab_size"]),
            max_position_embeddings=int(d["max_position_embeddings"]),
            type_vocab_size=int(d.get("type_vocab_size", 2)),
            layer_norm_eps=float(d.get("layer_norm_eps", 1e-12)),
        )

    def to_dict(self) -> dict:
        return {
            "model_type": "bert",
            "hidden_size": self.hidden_size,
            "num_hidden_layers": self.num_hidden_layers,
            "num_attention_heads": self.num_attention_heads,
            "intermediate_size": self.intermediate_size,
            "vocab_size": self.vocab_size,
            "max_position_embeddings": self.max_position_embeddings,
            "type_vocab_size": self.type_vocab_size,
            "layer_norm_eps": self.layer_norm_eps,
        }


def weight_prefix(weights: dict) -> str:
    """The ``"bert."`` prefix probe of ``BertBuilder::build`` (bert.rs:508-517)."""
    return "bert." if "bert.embeddings.word_embeddings.weight" in weights else ""


def layer_norm(x, gamma, beta, eps):
    """``(x - mean) / sqrt(var + eps) * gamma + beta`` over the last dim
    (layer_norm.rs:67-84; the fused eval path :55-65 is the same formula)."""
    mean = x.mean(axis=-1, keepdims=True)
    c = x - mean
    var = (c * c).mean(axis=-1, keepdims=True)
    return c / np.sqrt(var + eps) * gamma + beta


def linear(x, w, b=None):
    """``candle_nn::Linear``: ``x W^T + b`` with ``W`` stored ``[out, in]``."""
    y = x @ w.T
    return y if b is None else y + b


def gelu_erf(x):
    """``Tensor::gelu_erf``: ``0.5 x (1 + erf(x / sqrt 2))`` (bert.rs:189)."""
    return 0.5 * x * (1.0 + _erf(x / math.sqrt(2.0)))


def extended_attention_mask(mask):
    """``[B,S]`` {0,1} -> ``[B,1,1,S]`` additive: ``m*10000 - 10000`` (mask.rs:14-20)."""
    m = mask.astype(np.float32)
    return (m * np.float32(10000.0) - np.float32(10000.0))[:, None, None, :]


def softmax_last(x):
    m = x.max(axis=-1, keepdims=True)
    e = np.exp(x - m)
    return e / e.sum(axis=-1, keepdims=True)


def _w(weights, key, dtype):
    return np.asarray(weights[key], dtype=dtype)


LORA_SITES = ("query", "key", "value", "dense", "intermediate_dense", "output_dense")


def bert_forward_hidden(weights: dict, cfg: BertConfig, input_ids, mask,
                        dtype=np.float64, lora=None):
    """``Bert::forward_hidden`` (bert.rs:257-276) -> ``[B, S, H]``.

    ``lora``: optional ``{(layer, site): (A [rank, in], B [out, rank], scaling)}``
    over the six sites of ``lora_sites`` (bert.rs:437-446): each adapted linear
    is ``MaybeLoraLinear::Lora`` (crates/jammi-lora/src/wrapper.rs:15-42), whose
    inference forward is ``base(x) + scaling * (x @ A^T) @ B^T``
    (crates/jammi-lora/src/lora_linear.rs:226-305, no dropout)."""
    ids = np.asarray(input_ids, dtype=np.int64)
    mask = np.asarray(mask)
    B, S = ids.shape
    if S > cfg.max_position_embeddings:
        raise SequenceTooLong(f"sequence length {S} exceeds max {cfg.max_position_embeddings}")
    p = weight_prefix(weights)
    H, nh = cfg.hidden_size, cfg.num_attention_heads
    d = H // nh
    eps = cfg.layer_norm_eps
    g = lambda k: _w(weights, p + k, dtype)

    # BertEmbeddings::forward (bert.rs:102-111): token_type_ids are zeros (:269)
    x = g("embeddings.word_embeddings.weight")[ids]
    x = x + g("embeddings.token_type_embeddings.weight")[0]
    x = x + g("embeddings.position_embeddings.weight")[:S][None]
    x = layer_norm(x, g("embeddings.LayerNorm.weight"), g("embeddings.LayerNorm.bias"), eps)

    ext = extended_attention_mask(mask).astype(dtype)
    lora = lora or {}

    def lin(n, site, inp, name):
        y = linear(inp, g(pre + name + ".weight"), g(pre + name + ".bias"))
        if (n, site) in lora:
            a, b, scaling = lora[(n, site)]
            y = y + scaling * ((inp @ np.asarray(a, dtype).T) @ np.asarray(b, dtype).T)
        return y

    for n in range(cfg.num_hidden_layers):
        pre = f"encoder.layer.{n}."
        q = lin(n, "query", x, "attention.self.query")
        k = lin(n, "key", x, "attention.self.key")
        v = lin(n, "value", x, "attention.self.value")
        # transpose_for_scores (bert.rs:126-133): [B,S,H] -> [B,h,S,d]
        q = q.reshape(B, S, nh, d).transpose(0, 2, 1, 3)
        k = k.reshape(B, S, nh, d).transpose(0, 2, 1, 3)
        v = v.reshape(B, S, nh, d).transpose(0, 2, 1, 3)
        scores = (q @ k.transpose(0, 1, 3, 2)) / math.sqrt(d)
        probs = softmax_last(scores + ext)
        ctx = (probs @ v).transpose(0, 2, 1, 3).reshape(B, S, H)
        a = lin(n, "dense", ctx, "attention.output.dense")
        x1 = layer_norm(a + x, g(pre + "attention.output.LayerNorm.weight"),
                        g(pre + "attention.output.LayerNorm.bias"), eps)
        f = gelu_erf(lin(n, "intermediate_dense", x1, "intermediate.dense"))
        o = lin(n, "output_dense", f, "output.dense")
        x = layer_norm(o + x1, g(pre + "output.LayerNorm.weight"), g(pre + "output.LayerNorm.bias"), eps)
    return x


# ── pooling.rs ───────────────────────────────────────────────────────────────

def pool(hidden, mask, strategy=POOL_MEAN):
    """The four strategies of ``pool_and_normalize`` before L2 (pooling.rs:31-121)."""
    hidden = np.asarray(hidden)
    m = np.asarray(mask).astype(hidden.dtype)[:, :, None]
    if strategy == POOL_MEAN:  # pooling.rs:52-66, divisor floored at 1.0
        cnt = np.maximum(m.sum(axis=1), 1.0)
        return (hidden * m).sum(axis=1) / cnt
    if strategy == POOL_CLS:  # pooling.rs:68-70
        return hidden[:, 0, :]
    if strategy == POOL_MAX:  # pooling.rs:72-89, finite -1e30 sentinel at padding
        sent = np.asarray(-1e30, dtype=hidden.dtype)
        return np.where(m > 0, hidden, sent).max(axis=1)
    if strategy == POOL_WEIGHTED_MEAN:  # pooling.rs:103-121, 1-indexed position weights
        S = hidden.shape[1]
        w = np.arange(1, S + 1, dtype=hidden.dtype)[None, :, None] * m
        den = np.maximum(w.sum(axis=1), 1.0)
        return (hidden * w).sum(axis=1) / den
    raise ValueError(f"unknown pooling strategy {strategy}")


def l2_normalize(pooled, floor=1e-12):
    """``x / clamp(||x||, 1e-12, f32::MAX)`` (pooling.rs:123-139, 143-148).

    The squared norm is formed in float32 when the input is float32, so an
    all-padding max-pool row (-1e30 sentinel) overflows to inf and the clamp
    at ``f32::MAX`` engages, as it does in the reference.
    """
    pooled = np.asarray(pooled)
    fmax = np.finfo(np.float32).max
    with np.errstate(over="ignore"):
        sq = (pooled * pooled).sum(axis=-1, keepdims=True)
    # the reference squares and sums in f32: a sum beyond f32::MAX is inf
    norm = np.where(sq > fmax, np.inf, np.sqrt(sq))
    norm = np.clip(norm, floor, fmax)
    return pooled / norm


def pool_and_normalize(hidden, mask, strategy=POOL_MEAN):
    """``pool_and_normalize`` (pooling.rs:31-43)."""
    return l2_normalize(pool(hidden, mask, strategy))


def bert_forward(weights, cfg, input_ids, mask, strategy=POOL_MEAN, dtype=np.float64):
    """``Bert::forward`` (bert.rs:279-282): pooled, L2-normalised ``[B, H]``."""
    h = bert_forward_hidden(weights, cfg, input_ids, mask, dtype=dtype)
    return pool_and_normalize(h, mask, strategy)


# ── seeded synthetic fixtures ────────────────────────────────────────────────

def random_bert_weights(cfg: BertConfig, seed: int, std: float = 0.02,
                        dtype=np.float32) -> dict:
    """Random-init weights N(0, std), LayerNorm gain 1 / bias 0, biases 0 --
    the recipe of ``tests/fixtures/generate_tiny_bert.py`` in the reference,
    made reproducible by a seed.  HF key names, no prefix."""
    rng = np.random.default_rng(seed)
    H, F = cfg.hidden_size, cfg.intermediate_size
    r = lambda *s: (rng.standard_normal(s, dtype=np.float32) * std).astype(dtype)
    z = lambda n: np.zeros((n,), dtype=dtype)
    o = lambda n: np.ones((n,), dtype=dtype)
    w = {
        "embeddings.word_embeddings.weight": r(cfg.vocab_size, H),
        "embeddings.position_embeddings.weight": r(cfg.max_position_embeddings, H),
        "embeddings.token_type_embeddings.weight": r(cfg.type_vocab_size, H),
        "embeddings.LayerNorm.weight": o(H),
        "embeddings.LayerNorm.bias": z(H),
    }
    for n in range(cfg.num_hidden_layers):
        p = f"encoder.layer.{n}."
        for name in ("query", "key", "value"):
            w[p + f"attention.self.{name}.weight"] = r(H, H)
            w[p + f"attention.self.{name}.bias"] = z(H)
        w[p + "attention.output.dense.weight"] = r(H, H)
        w[p + "attention.output.dense.bias"] = z(H)
        w[p + "attention.output.LayerNorm.weight"] = o(H)
        w[p + "attention.output.LayerNorm.bias"] = z(H)
        w[p + "intermediate.dense.weight"] = r(F, H)
        w[p + "intermediate.dense.bias"] = z(F)
        w[p + "output.dense.weight"] = r(H, F)
        w[p + "output.dense.bias"] = z(H)
        w[p + "output.LayerNorm.weight"] = o(H)
        w[p + "output.LayerNorm.bias"] = z(H)
    return w


def random_token_batch(batch: int, seq: int, lengths, seed: int,
                       id_lo: int = 1000, id_hi: int = 30521,
                       cls_id: int = 101, sep_id: int = 102):
    """Token ids uniform in [id_lo, id_hi], [CLS] first, [SEP] at each row's
    end, zero padding and a {0,1} mask -- the layout ``BatchEncoding`` carries
    (crates/jammi-ai/src/model/tokenizer.rs:82-93, right padding)."""
    rng = np.random.default_rng(seed)
    ids = np.zeros((batch, seq), dtype=np.uint32)
    mask = np.zeros((batch, seq), dtype=np.uint32)
    for b, n in enumerate(lengths):
        n = int(n)
        if n <= 0:
            continue
        row = rng.integers(id_lo, id_hi + 1, size=n, dtype=np.int64)
        row[0] = cls_id
        if n > 1:
            row[n - 1] = sep_id
        ids[b, :n] = row
        mask[b, :n] = 1
    return ids, mask


def projection_head(x, lora_a, lora_b, lora_alpha):
    """Post-pool projection head of a fine-tuned embedding adapter: CandleModel
    applies it to the pooled, L2-normalised embedding without re-normalising
    (crates/jammi-ai/src/model/backend/candle.rs:823-829); load_projection_head
    (candle.rs:1857-1892) builds a LoraLinear over an identity base with
    scaling alpha / rank (crates/jammi-lora/src/lora_linear.rs:206-218), whose
    inference forward is base(x) + scaling * (x @ A^T) @ B^T (lora_linear.rs:226-305)."""
    x = np.asarray(x, dtype=np.float64)
    a = np.asarray(lora_a, dtype=np.float64)
    b = np.asarray(lora_b, dtype=np.float64)
    return x + (lora_alpha / a.shape[0]) * ((x @ a.T) @ b.T)


# ── DistilBERT ───────────────────────────────────────────────────────────────
# crates/jammi-encoders/src/distilbert.rs: the same post-LN encoder as BERT
# (embeddings :69-77 word + position then LayerNorm, no token-type table;
# attention :104-128 with the same additive mask; FFN :137-141 lin1 ->
# gelu_erf -> lin2; layer :152-162 residual then LayerNorm; forward_hidden
# :203-222), under its own config keys and weight names.
DISTILBERT_LAYER_NAMES = {  # DistilBERT module -> the BERT module computing the same op
    "attention.q_lin": "attention.self.query", "attention.k_lin": "attention.self.key",
    "attention.v_lin": "attention.self.value", "attention.out_lin": "attention.output.dense",
    "sa_layer_norm": "attention.output.LayerNorm", "ffn.lin1": "intermediate.dense",
    "ffn.lin2": "output.dense", "output_layer_norm": "output.LayerNorm",
}


def distilbert_config(d: dict) -> BertConfig:
    """``DistilBertConfig`` (distilbert.rs:32-57): dim / n_layers / n_heads /
    hidden_dim, layer_norm_eps default 1e-12, no token types."""
    return BertConfig(hidden_size=int(d["dim"]), num_hidden_layers=int(d["n_layers"]),
                      num_attention_heads=int(d["n_heads"]), intermediate_size=int(d["hidden_dim"]),
                      vocab_size=int(d["vocab_size"]),
                      max_position_embeddings=int(d["max_position_embeddings"]),
                      type_vocab_size=1, layer_norm_eps=float(d.get("layer_norm_eps", 1e-12)))


def distilbert_as_bert(weights: dict, d_cfg: dict):
    """DistilBERT weights (``distilbert.`` prefix, distilbert.rs:440) renamed onto
    the BERT modules that compute the same ops, with an all-zero token-type row
    (DistilBERT adds none): ``(bert_weights, BertConfig)``."""
    cfg = distilbert_config(d_cfg)
    w = {}
    for k, v in weights.items():
        k = k[len("distilbert."):] if k.startswith("distilbert.") else k
        if k.startswith("transformer.layer."):
            n, rest = k[len("transformer.layer."):].split(".", 1)
            for a, b in DISTILBERT_LAYER_NAMES.items():
                if rest.startswith(a + "."):
                    rest = b + rest[len(a):]
                    break
            k = f"encoder.layer.{n}.{rest}"
        w[k] = v
    w["embeddings.token_type_embeddings.weight"] = np.zeros((1, cfg.hidden_size))
    return w, cfg


DISTILBERT_LORA_SITES = ("q_lin", "k_lin", "v_lin", "out_lin", "lin1", "lin2")


def distilbert_forward_hidden(weights: dict, d_cfg: dict, input_ids, mask, dtype=np.float64,
                              lora=None):
    """``DistilBert::forward_hidden`` (distilbert.rs:203-222) -> ``[B, S, H]``.
    ``lora`` keys name DistilBERT's modules (``DISTILBERT_LORA_SITES``,
    distilbert.rs:245-296), mapped onto the same six sites."""
    w, cfg = distilbert_as_bert(weights, d_cfg)
    if lora:
        ren = dict(zip(DISTILBERT_LORA_SITES, LORA_SITES))
        lora = {(n, ren.get(s, s)): v for (n, s), v in lora.items()}
    return bert_forward_hidden(w, cfg, input_ids, mask, dtype=dtype, lora=lora)


# ── ModernBERT (crates/jammi-encoders/src/modernbert.rs) ─────────────────────

def modernbert_config(cfg: dict) -> dict:
    """``ModernBertConfig`` (modernbert.rs:72-90): the serde defaults for the
    optional fields (layer_norm_eps 1e-5, global_rope_theta 160000)."""
    return {
        "hidden_size": int(cfg["hidden_size"]), "num_hidden_layers": int(cfg["num_hidden_layers"]),
        "num_attention_heads": int(cfg["num_attention_heads"]),
        "intermediate_size": int(cfg["intermediate_size"]), "vocab_size": int(cfg["vocab_size"]),
        "max_position_embeddings": int(cfg["max_position_embeddings"]),
        "layer_norm_eps": float(cfg.get("layer_norm_eps", 1e-5)),
        "global_rope_theta": float(cfg.get("global_rope_theta", 160000.0)),
    }


def modernbert_rope_tables(head_dim: int, max_pos: int, base: float):
    """``RotaryEmbedding::new`` (modernbert.rs:106-131): theta = pos *
    base^(-2i/d) in float64, cos / sin stored as float32, ``[max_pos, d/2]``
    (the reference duplicates the halves to ``[max_pos, d]``)."""
    i = np.arange(head_dim // 2, dtype=np.float64)
    inv = np.power(float(base), -2.0 * i / head_dim)
    theta = np.arange(max_pos, dtype=np.float64)[:, None] * inv[None, :]
    return np.cos(theta).astype(np.float32), np.sin(theta).astype(np.float32)


def rope_apply(x, cos_half, sin_half):
    """``RotaryEmbedding::apply`` (modernbert.rs:133-163) on ``[B, h, S, d]``:
    ``x * cos + rotate_half(x) * sin``, ``rotate_half(x) = cat(-x2, x1)``."""
    half = x.shape[-1] // 2
    c = np.concatenate([cos_half, cos_half], axis=-1)[None, None]
    s = np.concatenate([sin_half, sin_half], axis=-1)[None, None]
    rot = np.concatenate([-x[..., half:], x[..., :half]], axis=-1)
    return x * c + rot * s


def modernbert_forward_hidden(weights: dict, cfg: dict, input_ids, mask, dtype=np.float64):
    """``ModernBert::forward_hidden`` (modernbert.rs:318-340) -> ``[B, S, H]``:
    embedding norm, then per layer the pre-norm attention with RoPE on Q and K
    (:178-227; layer 0 has no ``attn_norm``) and the GeGLU MLP
    ``Wo(gelu_erf(gate) * up)`` with gate the first half of ``Wi``'s output
    (:241-254), each added to its input; ``final_norm`` last.  LayerNorms carry
    no bias; linears carry none."""
    c = modernbert_config(cfg)
    H, L, nh, I = c["hidden_size"], c["num_hidden_layers"], c["num_attention_heads"], c["intermediate_size"]
    d = H // nh
    eps = c["layer_norm_eps"]
    p = "model." if "model.embeddings.tok_embeddings.weight" in weights else ""
    g = lambda k: np.asarray(weights[p + k], dtype=dtype)
    ids = np.asarray(input_ids, dtype=np.int64)
    mask = np.asarray(mask)
    B, S = ids.shape
    if S > c["max_position_embeddings"]:
        raise SequenceTooLong(S, c["max_position_embeddings"])
    zero = np.zeros((H,), dtype=dtype)
    x = layer_norm(g("embeddings.tok_embeddings.weight")[ids], g("embeddings.norm.weight"), zero, eps)
    ext = extended_attention_mask(mask).astype(dtype)
    cos, sin = modernbert_rope_tables(d, c["max_position_embeddings"], c["global_rope_theta"])
    cos, sin = cos[:S].astype(dtype), sin[:S].astype(dtype)
    for n in range(L):
        q_ = f"layers.{n}."
        h = x if n == 0 else layer_norm(x, g(q_ + "attn_norm.weight"), zero, eps)
        qkv = linear(h, g(q_ + "attn.Wqkv.weight"))
        q = qkv[..., :H].reshape(B, S, nh, d).transpose(0, 2, 1, 3)
        k = qkv[..., H:2 * H].reshape(B, S, nh, d).transpose(0, 2, 1, 3)
        v = qkv[..., 2 * H:].reshape(B, S, nh, d).transpose(0, 2, 1, 3)
        q, k = rope_apply(q, cos, sin), rope_apply(k, cos, sin)
        probs = softmax_last((q @ k.transpose(0, 1, 3, 2)) / math.sqrt(d) + ext)
        ctx = (probs @ v).transpose(0, 2, 1, 3).reshape(B, S, H)
        x = x + linear(ctx, g(q_ + "attn.Wo.weight"))
        h = layer_norm(x, g(q_ + "mlp_norm.weight"), zero, eps)
        ug = linear(h, g(q_ + "mlp.Wi.weight"))
        x = x + linear(gelu_erf(ug[..., :I]) * ug[..., I:], g(q_ + "mlp.Wo.weight"))
    return layer_norm(x, g("final_norm.weight"), zero, eps)


def random_modernbert_weights(cfg: dict, seed: int, std: float = 0.02, dtype=np.float32) -> dict:
    """Random-init ModernBERT weights under the reference's ``model.`` keys
    (modernbert.rs:16-27): N(0, std), LayerNorm weights 1 +- 0.1 noise."""
    c = modernbert_config(cfg)
    rng = np.random.default_rng(seed)
    H, I = c["hidden_size"], c["intermediate_size"]
    r = lambda *s: (rng.standard_normal(s, dtype=np.float32) * std).astype(dtype)
    ln = lambda: (1.0 + 0.1 * rng.standard_normal(H, dtype=np.float32)).astype(dtype)
    w = {"model.embeddings.tok_embeddings.weight": r(c["vocab_size"], H),
         "model.embeddings.norm.weight": ln(), "model.final_norm.weight": ln()}
    for n in range(c["num_hidden_layers"]):
        q = f"model.layers.{n}."
        if n > 0:
            w[q + "attn_norm.weight"] = ln()
        w[q + "attn.Wqkv.weight"] = r(3 * H, H)
        w[q + "attn.Wo.weight"] = r(H, H)
        w[q + "mlp_norm.weight"] = ln()
        w[q + "mlp.Wi.weight"] = r(2 * I, H)
        w[q + "mlp.Wo.weight"] = r(H, I)
    return w
