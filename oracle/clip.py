"""numpy restatement of the reference OpenCLIP vision tower (test oracle only).

Follows ``crates/jammi-ai/src/model/backend/open_clip_vit.rs``:

* ``quick_gelu``                   :123-125  ``x * sigmoid(1.702 x)``
* ``MultiHeadAttention::forward``  :151-180  fused in_proj, unmasked softmax
* ``Mlp::forward``                 :196-200
* ``ResidualAttentionBlock``       :226-236  pre-LN (eps 1e-5), two residuals
* ``OpenClipVisionTransformer::forward`` :309-353  conv1 (kernel = stride =
  patch, no bias) -> CLS cat -> +pos -> ln_pre -> blocks -> CLS or GAP pool
  (:339-346) -> ln_post -> ``@ proj``
* the caller's ``l2_normalize``    crates/jammi-ai/src/model/backend/candle.rs:425-438

and the OpenCLIP text tower, ``crates/jammi-encoders/src/clip_text.rs``:

* ``ClipTextConfig::from_open_clip_config`` :53-102  (context 77, vocab 49408,
  heads width/64 by default; MLP width 4x, :195)
* ``ClipText::forward``            :296-331  token + positional embedding ->
  causally masked pre-LN blocks (:133-162, mask :350-362) -> ``ln_final`` ->
  the hidden state at ``argmax(input_ids)`` (the EOT token, :322-326) ->
  ``@ text_projection`` -> L2 (:379-389)
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np

from .bert import layer_norm, linear, softmax_last

CLIP_LN_EPS = 1e-5


@dataclass
class ClipVisionConfig:
    """``OpenClipVisionConfig`` (open_clip_vit.rs:19-41, parsed at :45-101)."""
    width: int = 768
    layers: int = 12
    heads: int = 12
    mlp_ratio: float = 4.0
    image_size: int = 224
    patch_size: int = 32
    embed_dim: int = 512
    global_average_pool: bool = False

    @property
    def grid(self) -> int:
        return self.image_size // self.patch_size

    @property
    def tokens(self) -> int:
        return self.grid * self.grid + 1

    @property
    def mlp(self) -> int:
        return int(self.width * self.mlp_ratio)

    @classmethod
    def from_open_clip_config(cls, d: dict) -> "ClipVisionConfig":
        mc = d["model_cfg"]
        vc = mc["vision_cfg"]
        width = int(vc.get("width", 768))
        return cls(
            width=width,
            layers=int(vc.get("layers", 12)),
            heads=int(vc.get("heads", width // 64)),
            mlp_ratio=float(vc.get("mlp_ratio", 4.0)),
            image_size=int(vc.get("image_size", 224)),
            patch_size=int(vc.get("patch_size", 32)),
            embed_dim=int(mc["embed_dim"]),
            global_average_pool=bool(vc.get("global_average_pool", False)),
        )

    def to_open_clip_config(self) -> dict:
        return {"model_cfg": {"embed_dim": self.embed_dim, "vision_cfg": {
            "image_size": self.image_size, "patch_size": self.patch_size,
            "width": self.width, "layers": self.layers, "heads": self.heads,
            "mlp_ratio": self.mlp_ratio,
            "global_average_pool": self.global_average_pool}}}


def quick_gelu(x):
    return x * (1.0 / (1.0 + np.exp(-1.702 * x)))


def patchify(pixels, patch):
    """conv1 as a matmul operand: ``[B,3,I,I] -> [B, g*g, 3*p*p]`` with the
    (channel, ky, kx) order of the conv weight ``[W, 3, p, p]``, patches in
    row-major grid order (the ``flatten_from(2).permute(0,2,1)`` of :316)."""
    B, C, I, _ = pixels.shape
    g = I // patch
    x = pixels.reshape(B, C, g, patch, g, patch)
    x = x.transpose(0, 2, 4, 1, 3, 5)  # B, gy, gx, C, ky, kx
    return x.reshape(B, g * g, C * patch * patch)


def clip_vision_forward(weights: dict, cfg: ClipVisionConfig, pixels,
                        dtype=np.float64, prefix: str = "visual."):
    """``OpenClipVisionTransformer::forward`` -> un-normalised ``[B, embed_dim]``."""
    g = lambda k: np.asarray(weights[prefix + k], dtype=dtype)
    px = np.asarray(pixels, dtype=dtype)
    B = px.shape[0]
    W, nh = cfg.width, cfg.heads
    d = W // nh
    conv = g("conv1.weight").reshape(W, -1)
    x = patchify(px, cfg.patch_size) @ conv.T                       # [B, g*g, W]
    cls = np.broadcast_to(g("class_embedding")[None, None, :], (B, 1, W))
    x = np.concatenate([cls, x], axis=1) + g("positional_embedding")[None]
    x = layer_norm(x, g("ln_pre.weight"), g("ln_pre.bias"), CLIP_LN_EPS)
    T = x.shape[1]
    for i in range(cfg.layers):
        p = f"transformer.resblocks.{i}."
        h = layer_norm(x, g(p + "ln_1.weight"), g(p + "ln_1.bias"), CLIP_LN_EPS)
        qkv = linear(h, g(p + "attn.in_proj_weight"), g(p + "attn.in_proj_bias"))
        qkv = qkv.reshape(B, T, 3, nh, d).transpose(2, 0, 3, 1, 4)
        q, k, v = qkv[0], qkv[1], qkv[2]
        a = softmax_last((q @ k.transpose(0, 1, 3, 2)) / math.sqrt(d)) @ v
        a = a.transpose(0, 2, 1, 3).reshape(B, T, W)
        x = x + linear(a, g(p + "attn.out_proj.weight"), g(p + "attn.out_proj.bias"))
        h = layer_norm(x, g(p + "ln_2.weight"), g(p + "ln_2.bias"), CLIP_LN_EPS)
        h = quick_gelu(linear(h, g(p + "mlp.c_fc.weight"), g(p + "mlp.c_fc.bias")))
        x = x + linear(h, g(p + "mlp.c_proj.weight"), g(p + "mlp.c_proj.bias"))
    pooled = x[:, 1:, :].mean(axis=1) if cfg.global_average_pool else x[:, 0, :]
    pooled = layer_norm(pooled, g("ln_post.weight"), g("ln_post.bias"), CLIP_LN_EPS)
    return pooled @ g("proj")


def l2_normalize_image(x):
    """``l2_normalize`` of the image path: ``x / clamp(||x||, 1e-12)`` (candle.rs:425-438)."""
    n = np.sqrt((x * x).sum(axis=-1, keepdims=True))
    return x / np.maximum(n, 1e-12)


def random_clip_weights(cfg: ClipVisionConfig, seed: int, std: float = 0.02,
                        dtype=np.float32, prefix: str = "visual.") -> dict:
    """Random-init OpenCLIP ``visual.*`` weights N(0, std), LN gain 1 / bias 0."""
    rng = np.random.default_rng(seed)
    W, F, P = cfg.width, cfg.mlp, cfg.patch_size
    r = lambda *s: (rng.standard_normal(s, dtype=np.float32) * std).astype(dtype)
    z = lambda n: np.zeros((n,), dtype=dtype)
    o = lambda n: np.ones((n,), dtype=dtype)
    w = {
        "conv1.weight": r(W, 3, P, P),
        "class_embedding": r(W),
        "positional_embedding": r(cfg.tokens, W),
        "ln_pre.weight": o(W), "ln_pre.bias": z(W),
        "ln_post.weight": o(W), "ln_post.bias": z(W),
        "proj": r(W, cfg.embed_dim),
    }
    for i in range(cfg.layers):
        p = f"transformer.resblocks.{i}."
        w[p + "ln_1.weight"] = o(W); w[p + "ln_1.bias"] = z(W)
        w[p + "ln_2.weight"] = o(W); w[p + "ln_2.bias"] = z(W)
        w[p + "attn.in_proj_weight"] = r(3 * W, W)
        w[p + "attn.in_proj_bias"] = r(3 * W)
        w[p + "attn.out_proj.weight"] = r(W, W)
        w[p + "attn.out_proj.bias"] = r(W)
        w[p + "mlp.c_fc.weight"] = r(F, W)
        w[p + "mlp.c_fc.bias"] = r(F)
        w[p + "mlp.c_proj.weight"] = r(W, F)
        w[p + "mlp.c_proj.bias"] = r(W)
    return {prefix + k: v for k, v in w.items()}


# ── OpenCLIP text tower (clip_text.rs) ───────────────────────────────────────

@dataclass
class ClipTextConfig:
    """``ClipTextConfig`` (clip_text.rs:30-45, parsed at :53-102)."""
    width: int = 512
    layers: int = 12
    heads: int = 8
    context_length: int = 77
    vocab_size: int = 49408
    embed_dim: int = 512

    @property
    def mlp(self) -> int:
        return 4 * self.width  # fixed 4x MLP ratio (clip_text.rs:194-195)

    @classmethod
    def from_open_clip_config(cls, d: dict) -> "ClipTextConfig":
        mc = d["model_cfg"]
        tc = mc["text_cfg"]
        width = int(tc["width"])
        return cls(width=width, layers=int(tc["layers"]), heads=int(tc.get("heads", width // 64)),
                   context_length=int(tc.get("context_length", 77)),
                   vocab_size=int(tc.get("vocab_size", 49408)), embed_dim=int(mc["embed_dim"]))

    def to_open_clip_config(self) -> dict:
        return {"model_cfg": {"embed_dim": self.embed_dim, "text_cfg": {
            "context_length": self.context_length, "vocab_size": self.vocab_size,
            "width": self.width, "layers": self.layers, "heads": self.heads}}}


def clip_text_forward(weights: dict, cfg: ClipTextConfig, input_ids, dtype=np.float64):
    """``ClipText::forward`` (clip_text.rs:296-331) -> L2-normalised ``[B, embed_dim]``.

    The causal mask adds ``f32::MIN`` above the diagonal (:350-362), whose
    exponential is exactly 0: keys after the query are excluded.  Pooling takes
    the first position of the row's largest id (``argmax``, :322-326)."""
    g = lambda k: np.asarray(weights[k], dtype=dtype)
    ids = np.asarray(input_ids, dtype=np.int64)
    B, S = ids.shape
    if S > cfg.context_length:
        raise ValueError(f"sequence length {S} exceeds context length {cfg.context_length}")
    W, nh = cfg.width, cfg.heads
    d = W // nh
    x = g("token_embedding.weight")[ids] + g("positional_embedding")[:S][None]
    causal = np.triu(np.ones((S, S), dtype=bool), k=1)
    for i in range(cfg.layers):
        p = f"transformer.resblocks.{i}."
        h = layer_norm(x, g(p + "ln_1.weight"), g(p + "ln_1.bias"), CLIP_LN_EPS)
        qkv = linear(h, g(p + "attn.in_proj_weight"), g(p + "attn.in_proj_bias"))
        qkv = qkv.reshape(B, S, 3, nh, d).transpose(2, 0, 3, 1, 4)
        q, k, v = qkv[0], qkv[1], qkv[2]
        sc = (q @ k.transpose(0, 1, 3, 2)) / math.sqrt(d)
        sc = np.where(causal[None, None], -np.inf, sc)
        a = softmax_last(sc) @ v
        a = a.transpose(0, 2, 1, 3).reshape(B, S, W)
        x = x + linear(a, g(p + "attn.out_proj.weight"), g(p + "attn.out_proj.bias"))
        h = layer_norm(x, g(p + "ln_2.weight"), g(p + "ln_2.bias"), CLIP_LN_EPS)
        h = quick_gelu(linear(h, g(p + "mlp.c_fc.weight"), g(p + "mlp.c_fc.bias")))
        x = x + linear(h, g(p + "mlp.c_proj.weight"), g(p + "mlp.c_proj.bias"))
    x = layer_norm(x, g("ln_final.weight"), g("ln_final.bias"), CLIP_LN_EPS)
    eot = ids.argmax(axis=1)
    pooled = x[np.arange(B), eot]
    return l2_normalize_image(pooled @ g("text_projection"))


def random_clip_text_weights(cfg: ClipTextConfig, seed: int, std: float = 0.02,
                             dtype=np.float32) -> dict:
    """Random-init OpenCLIP text weights (root-level keys) N(0, std), LN gain 1 / bias 0."""
    rng = np.random.default_rng(seed)
    W, F = cfg.width, cfg.mlp
    r = lambda *s: (rng.standard_normal(s, dtype=np.float32) * std).astype(dtype)
    z = lambda n: np.zeros((n,), dtype=dtype)
    o = lambda n: np.ones((n,), dtype=dtype)
    w = {
        "token_embedding.weight": r(cfg.vocab_size, W),
        "positional_embedding": r(cfg.context_length, W),
        "ln_final.weight": o(W), "ln_final.bias": z(W),
        "text_projection": r(W, cfg.embed_dim),
    }
    for i in range(cfg.layers):
        p = f"transformer.resblocks.{i}."
        w[p + "ln_1.weight"] = o(W); w[p + "ln_1.bias"] = z(W)
        w[p + "ln_2.weight"] = o(W); w[p + "ln_2.bias"] = z(W)
        w[p + "attn.in_proj_weight"] = r(3 * W, W)
        w[p + "attn.in_proj_bias"] = r(3 * W)
        w[p + "attn.out_proj.weight"] = r(W, W)
        w[p + "attn.out_proj.bias"] = r(W)
        w[p + "mlp.c_fc.weight"] = r(F, W)
        w[p + "mlp.c_fc.bias"] = r(F)
        w[p + "mlp.c_proj.weight"] = r(W, F)
        w[p + "mlp.c_proj.bias"] = r(W)
    return w


def random_clip_text_batch(batch: int, seq: int, lengths, seed: int, vocab: int):
    """OpenCLIP tokenizer layout: <|startoftext|> (vocab-2) first, text ids in
    [1, vocab-3], <|endoftext|> (vocab-1, the row's largest id) at position
    len-1, zeros after (clip_bpe.rs:170-200)."""
    rng = np.random.default_rng(seed)
    ids = np.zeros((batch, seq), dtype=np.uint32)
    for b, n in enumerate(lengths):
        n = int(n)
        assert 2 <= n <= seq
        ids[b, 0] = vocab - 2
        ids[b, 1:n - 1] = rng.integers(1, vocab - 2, size=n - 2)
        ids[b, n - 1] = vocab - 1
    return ids
