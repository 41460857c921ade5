"""Generate the golden fixtures under tests/golden/ (run once, here, on CPU).

    JAMMI_REFERENCE=<reference checkout> python tests/golden/make_golden.py

(``reference_tiny_bert.npz`` needs the reference checkout, named by the
JAMMI_REFERENCE environment variable; the other fixtures need nothing.)

Expected outputs come from HuggingFace ``transformers`` (``BertModel`` and
``CLIPVisionModelWithProjection``, eager attention, float64), an independent
implementation of the same encoder math that the reference's own parity test
(``crates/jammi-encoders/tests/parity.rs``) checks its encoder against through
candle-transformers.  Pooling and L2 are applied with torch ops following
``crates/jammi-encoders/src/pooling.rs`` -- written here independently of
``oracle/``, so the oracle can be pinned against these files.

Fixtures (``.npz``, weights included so the GPU tests need nothing else):

* ``tiny_bert_seeded.npz``    H 32, 1 layer, 2 heads, FFN 128, vocab 256, pos 128
  (the shape of the reference's ``cookbook/fixtures/tiny_bert``), seeded weights,
  ragged rows including a one-token row and an all-padding row.
* ``small_bert_prefixed.npz`` H 64, 2 layers, 4 heads, FFN 256, keys under the
  ``bert.`` prefix (the ``BertForX`` layout probed at ``bert.rs:508-517``).
* ``tiny_clip_gap.npz`` / ``tiny_clip_cls.npz``  OpenCLIP ViT W 32, 1 layer,
  4 heads, patch 4, image 8, embed 16 (the shape of the reference's
  ``tests/fixtures/tiny_open_clip``), global-average and CLS pooling.
* ``small_clip_text.npz``  OpenCLIP text tower W 64, 2 layers, context 24 (HF
  ``CLIPTextModelWithProjection``, float64), ragged EOT positions.
* ``small_modernbert.npz``  ModernBERT (HF ``ModernBertModel``, every layer global) H 64,
  3 layers, 4 heads, GeGLU 96, RoPE theta 160000, keys under ``model.``
  (``crates/jammi-encoders/src/modernbert.rs``).
* ``small_distilbert.npz``  DistilBERT (HF ``DistilBertModel``) H 64, 2 layers, 4 heads,
  FFN 256: the BERT weight recipe under DistilBERT names (``distilbert.`` prefix,
  ``transformer.layer.N.{attention.q_lin, ..., ffn.lin1, output_layer_norm}``) and no
  token-type table (``crates/jammi-encoders/src/distilbert.rs``).
* ``reference_tiny_bert.npz`` outputs of the reference's own committed
  ``tiny_bert`` fixture (weights are NOT copied: its sha256 is stored and the
  CPU test re-reads the fixture when the reference checkout is present).
"""
from __future__ import annotations

import hashlib
import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.abspath(os.path.join(HERE, "..", "..")))

from oracle.bert import BertConfig, random_bert_weights  # noqa: E402  (weight recipe only)
from oracle.clip import (ClipTextConfig, ClipVisionConfig, random_clip_text_batch,  # noqa: E402
                         random_clip_text_weights, random_clip_weights)

REF_ROOT = os.environ.get("JAMMI_REFERENCE", "")
REF_TINY_BERT = os.path.join(REF_ROOT, "cookbook", "fixtures", "tiny_bert") if REF_ROOT else ""


def torch_pool_all(hidden: torch.Tensor, mask: torch.Tensor) -> dict:
    """pooling.rs:31-148 restated with torch ops (float64)."""
    m = mask.to(torch.float64).unsqueeze(-1)
    S = hidden.shape[1]
    out = {}
    out["mean"] = (hidden * m).sum(1) / m.sum(1).clamp(min=1.0)
    out["cls"] = hidden[:, 0, :]
    out["max"] = torch.where(m > 0, hidden, torch.full_like(hidden, -1e30)).amax(1)
    w = torch.arange(1, S + 1, dtype=torch.float64).view(1, S, 1) * m
    out["weighted_mean"] = (hidden * w).sum(1) / w.sum(1).clamp(min=1.0)
    res = {}
    for k, v in out.items():
        # the reference forms the norm in the compute dtype (f32 on CPU) and
        # clamps at f32::MAX; in float64 the clamp is a no-op except for the
        # max-pool all-padding row, handled identically by taking the f32 norm.
        n32 = torch.sqrt((v.to(torch.float32) ** 2).sum(-1, keepdim=True)).to(torch.float64)
        n = torch.sqrt((v ** 2).sum(-1, keepdim=True))
        n = torch.where(torch.isinf(n32), torch.full_like(n, float(np.finfo(np.float32).max)), n)
        res[k] = v / n.clamp(min=1e-12)
    return res


def hf_bert_hidden(weights: dict, cfg: BertConfig, ids, mask) -> np.ndarray:
    from transformers import BertConfig as HFBertConfig, BertModel
    hcfg = HFBertConfig(vocab_size=cfg.vocab_size, hidden_size=cfg.hidden_size,
                        num_hidden_layers=cfg.num_hidden_layers,
                        num_attention_heads=cfg.num_attention_heads,
                        intermediate_size=cfg.intermediate_size, hidden_act="gelu",
                        hidden_dropout_prob=0.0, attention_probs_dropout_prob=0.0,
                        max_position_embeddings=cfg.max_position_embeddings,
                        type_vocab_size=cfg.type_vocab_size,
                        layer_norm_eps=cfg.layer_norm_eps)
    hcfg._attn_implementation = "eager"
    model = BertModel(hcfg, add_pooling_layer=False).eval().to(torch.float64)
    sd = {k[5:] if k.startswith("bert.") else k: torch.from_numpy(np.asarray(v, dtype=np.float64))
          for k, v in weights.items()}
    missing, unexpected = model.load_state_dict(sd, strict=False)
    missing = [k for k in missing if not k.endswith("position_ids") and "token_type_ids" not in k]
    assert not missing and not unexpected, (missing, unexpected)
    with torch.no_grad():
        out = model(input_ids=torch.from_numpy(ids.astype(np.int64)),
                    attention_mask=torch.from_numpy(mask.astype(np.int64)),
                    token_type_ids=torch.zeros(ids.shape, dtype=torch.int64))
    return out.last_hidden_state.numpy()


def bert_fixture(name, cfg: BertConfig, seed, lens, S, prefix=""):
    w = random_bert_weights(cfg, seed)
    if prefix:
        w = {prefix + k: v for k, v in w.items()}
    rng = np.random.default_rng(seed + 1)
    B = len(lens)
    ids = np.zeros((B, S), dtype=np.uint32)
    mask = np.zeros((B, S), dtype=np.uint32)
    for b, n in enumerate(lens):
        ids[b, :n] = rng.integers(1, cfg.vocab_size, size=n)
        mask[b, :n] = 1
    hidden = hf_bert_hidden(w, cfg, ids, mask)
    pooled = torch_pool_all(torch.from_numpy(hidden), torch.from_numpy(mask.astype(np.int64)))
    arrs = {"w::" + k: v for k, v in w.items()}
    arrs.update({"ids": ids, "mask": mask, "hidden": hidden,
                 "config_json": np.frombuffer(json.dumps(cfg.to_dict()).encode(), dtype=np.uint8)})
    arrs.update({"pooled_" + k: v.numpy() for k, v in pooled.items()})
    np.savez_compressed(os.path.join(HERE, name), **arrs)
    print("wrote", name, {k: v.shape for k, v in arrs.items() if not k.startswith("w::")})


DISTIL_NAMES = {  # BERT recipe name -> DistilBERT name (distilbert.rs:440-545)
    "attention.self.query": "attention.q_lin", "attention.self.key": "attention.k_lin",
    "attention.self.value": "attention.v_lin", "attention.output.dense": "attention.out_lin",
    "attention.output.LayerNorm": "sa_layer_norm", "intermediate.dense": "ffn.lin1",
    "output.dense": "ffn.lin2", "output.LayerNorm": "output_layer_norm",
}


def distil_weights(cfg: BertConfig, seed) -> dict:
    """The BERT weight recipe under DistilBERT names (prefix ``distilbert.``,
    ``transformer.layer.N``), without the token-type table."""
    out = {}
    for k, v in random_bert_weights(cfg, seed).items():
        if "token_type_embeddings" in k:
            continue
        if k.startswith("encoder.layer."):
            n, rest = k[len("encoder.layer."):].split(".", 1)
            for a, b in DISTIL_NAMES.items():
                if rest.startswith(a + "."):
                    rest = b + rest[len(a):]
                    break
            k = f"transformer.layer.{n}.{rest}"
        out["distilbert." + k] = v
    return out


def hf_distilbert_hidden(weights: dict, cfg: BertConfig, ids, mask) -> np.ndarray:
    from transformers import DistilBertConfig, DistilBertModel
    hcfg = DistilBertConfig(vocab_size=cfg.vocab_size, dim=cfg.hidden_size,
                            n_layers=cfg.num_hidden_layers, n_heads=cfg.num_attention_heads,
                            hidden_dim=cfg.intermediate_size, activation="gelu", dropout=0.0,
                            attention_dropout=0.0,
                            max_position_embeddings=cfg.max_position_embeddings,
                            sinusoidal_pos_embds=False)
    hcfg._attn_implementation = "eager"
    model = DistilBertModel(hcfg).eval().to(torch.float64)
    sd = {k[len("distilbert."):]: torch.from_numpy(np.asarray(v, dtype=np.float64))
          for k, v in weights.items()}
    missing, unexpected = model.load_state_dict(sd, strict=False)
    missing = [k for k in missing if not k.endswith("position_ids")]
    assert not missing and not unexpected, (missing, unexpected)
    with torch.no_grad():
        out = model(input_ids=torch.from_numpy(ids.astype(np.int64)),
                    attention_mask=torch.from_numpy(mask.astype(np.int64)))
    return out.last_hidden_state.numpy()


def distilbert_fixture(name, cfg: BertConfig, seed, lens, S):
    w = distil_weights(cfg, seed)
    rng = np.random.default_rng(seed + 1)
    B = len(lens)
    ids = np.zeros((B, S), dtype=np.uint32)
    mask = np.zeros((B, S), dtype=np.uint32)
    for b, n in enumerate(lens):
        ids[b, :n] = rng.integers(1, cfg.vocab_size, size=n)
        mask[b, :n] = 1
    hidden = hf_distilbert_hidden(w, cfg, ids, mask)
    pooled = torch_pool_all(torch.from_numpy(hidden), torch.from_numpy(mask.astype(np.int64)))
    dcfg = {"model_type": "distilbert", "dim": cfg.hidden_size, "n_layers": cfg.num_hidden_layers,
            "n_heads": cfg.num_attention_heads, "hidden_dim": cfg.intermediate_size,
            "vocab_size": cfg.vocab_size, "max_position_embeddings": cfg.max_position_embeddings}
    arrs = {"w::" + k: v for k, v in w.items()}
    arrs.update({"ids": ids, "mask": mask, "hidden": hidden,
                 "config_json": np.frombuffer(json.dumps(dcfg).encode(), dtype=np.uint8)})
    arrs.update({"pooled_" + k: v.numpy() for k, v in pooled.items()})
    np.savez_compressed(os.path.join(HERE, name), **arrs)
    print("wrote", name, {k: v.shape for k, v in arrs.items() if not k.startswith("w::")})


def hf_clip_embed(w: dict, cfg: ClipVisionConfig, pixels) -> np.ndarray:
    from transformers import CLIPVisionConfig, CLIPVisionModelWithProjection
    hcfg = CLIPVisionConfig(hidden_size=cfg.width, intermediate_size=cfg.mlp,
                            num_hidden_layers=cfg.layers, num_attention_heads=cfg.heads,
                            image_size=cfg.image_size, patch_size=cfg.patch_size,
                            projection_dim=cfg.embed_dim, hidden_act="quick_gelu",
                            layer_norm_eps=1e-5, num_channels=3)
    hcfg._attn_implementation = "eager"
    model = CLIPVisionModelWithProjection(hcfg).eval().to(torch.float64)
    t = lambda k: torch.from_numpy(np.asarray(w["visual." + k], dtype=np.float64))
    W = cfg.width
    sd = {
        "vision_model.embeddings.class_embedding": t("class_embedding"),
        "vision_model.embeddings.patch_embedding.weight": t("conv1.weight"),
        "vision_model.embeddings.position_embedding.weight": t("positional_embedding"),
        "vision_model.pre_layrnorm.weight": t("ln_pre.weight"),
        "vision_model.pre_layrnorm.bias": t("ln_pre.bias"),
        "vision_model.post_layernorm.weight": t("ln_post.weight"),
        "vision_model.post_layernorm.bias": t("ln_post.bias"),
        "visual_projection.weight": t("proj").T.contiguous(),
    }
    for i in range(cfg.layers):
        p = f"transformer.resblocks.{i}."
        q = f"vision_model.encoder.layers.{i}."
        ipw, ipb = t(p + "attn.in_proj_weight"), t(p + "attn.in_proj_bias")
        for j, nm in enumerate(("q_proj", "k_proj", "v_proj")):
            sd[q + f"self_attn.{nm}.weight"] = ipw[j * W:(j + 1) * W]
            sd[q + f"self_attn.{nm}.bias"] = ipb[j * W:(j + 1) * W]
        sd[q + "self_attn.out_proj.weight"] = t(p + "attn.out_proj.weight")
        sd[q + "self_attn.out_proj.bias"] = t(p + "attn.out_proj.bias")
        sd[q + "layer_norm1.weight"] = t(p + "ln_1.weight")
        sd[q + "layer_norm1.bias"] = t(p + "ln_1.bias")
        sd[q + "layer_norm2.weight"] = t(p + "ln_2.weight")
        sd[q + "layer_norm2.bias"] = t(p + "ln_2.bias")
        sd[q + "mlp.fc1.weight"] = t(p + "mlp.c_fc.weight")
        sd[q + "mlp.fc1.bias"] = t(p + "mlp.c_fc.bias")
        sd[q + "mlp.fc2.weight"] = t(p + "mlp.c_proj.weight")
        sd[q + "mlp.fc2.bias"] = t(p + "mlp.c_proj.bias")
    missing, unexpected = model.load_state_dict(sd, strict=False)
    missing = [k for k in missing if "position_ids" not in k]
    assert not missing and not unexpected, (missing, unexpected)
    px = torch.from_numpy(np.asarray(pixels, dtype=np.float64))
    with torch.no_grad():
        if not cfg.global_average_pool:
            e = model(pixel_values=px).image_embeds
        else:
            vm = model.vision_model
            hs = vm.encoder(inputs_embeds=vm.pre_layrnorm(vm.embeddings(px))).last_hidden_state
            e = model.visual_projection(vm.post_layernorm(hs[:, 1:, :].mean(1)))
    e = e.numpy()
    return e, e / np.maximum(np.linalg.norm(e, axis=-1, keepdims=True), 1e-12)


def clip_fixture(name, cfg: ClipVisionConfig, seed, batch):
    w = random_clip_weights(cfg, seed)
    pixels = np.random.default_rng(seed + 1).standard_normal(
        (batch, 3, cfg.image_size, cfg.image_size)).astype(np.float32)
    raw, normed = hf_clip_embed(w, cfg, pixels)
    arrs = {"w::" + k: v for k, v in w.items()}
    arrs.update({"pixels": pixels, "embed_raw": raw, "embed": normed,
                 "config_json": np.frombuffer(json.dumps(cfg.to_open_clip_config()).encode(), dtype=np.uint8)})
    np.savez_compressed(os.path.join(HERE, name), **arrs)
    print("wrote", name, raw.shape)


def hf_clip_text_embed(w: dict, cfg: ClipTextConfig, ids) -> np.ndarray:
    """HF ``CLIPTextModelWithProjection`` in float64 over the OpenCLIP text
    weights: split ``in_proj``, ``text_projection`` transposed, quick-GELU, eps
    1e-5, ``eos_token_id`` 2 (pooling at ``argmax(input_ids)``), causal mask."""
    from transformers import CLIPTextConfig, CLIPTextModelWithProjection
    hcfg = CLIPTextConfig(vocab_size=cfg.vocab_size, hidden_size=cfg.width,
                          intermediate_size=cfg.mlp, projection_dim=cfg.embed_dim,
                          num_hidden_layers=cfg.layers, num_attention_heads=cfg.heads,
                          max_position_embeddings=cfg.context_length, hidden_act="quick_gelu",
                          layer_norm_eps=1e-5, eos_token_id=2)
    hcfg._attn_implementation = "eager"
    model = CLIPTextModelWithProjection(hcfg).eval().to(torch.float64)
    t = lambda k: torch.from_numpy(np.asarray(w[k], dtype=np.float64))
    W = cfg.width
    sd = {
        "text_model.embeddings.token_embedding.weight": t("token_embedding.weight"),
        "text_model.embeddings.position_embedding.weight": t("positional_embedding"),
        "text_model.final_layer_norm.weight": t("ln_final.weight"),
        "text_model.final_layer_norm.bias": t("ln_final.bias"),
        "text_projection.weight": t("text_projection").T.contiguous(),
    }
    for i in range(cfg.layers):
        p = f"transformer.resblocks.{i}."
        q = f"text_model.encoder.layers.{i}."
        ipw, ipb = t(p + "attn.in_proj_weight"), t(p + "attn.in_proj_bias")
        for j, nm in enumerate(("q_proj", "k_proj", "v_proj")):
            sd[q + f"self_attn.{nm}.weight"] = ipw[j * W:(j + 1) * W]
            sd[q + f"self_attn.{nm}.bias"] = ipb[j * W:(j + 1) * W]
        sd[q + "self_attn.out_proj.weight"] = t(p + "attn.out_proj.weight")
        sd[q + "self_attn.out_proj.bias"] = t(p + "attn.out_proj.bias")
        sd[q + "layer_norm1.weight"] = t(p + "ln_1.weight")
        sd[q + "layer_norm1.bias"] = t(p + "ln_1.bias")
        sd[q + "layer_norm2.weight"] = t(p + "ln_2.weight")
        sd[q + "layer_norm2.bias"] = t(p + "ln_2.bias")
        sd[q + "mlp.fc1.weight"] = t(p + "mlp.c_fc.weight")
        sd[q + "mlp.fc1.bias"] = t(p + "mlp.c_fc.bias")
        sd[q + "mlp.fc2.weight"] = t(p + "mlp.c_proj.weight")
        sd[q + "mlp.fc2.bias"] = t(p + "mlp.c_proj.bias")
    missing, unexpected = model.load_state_dict(sd, strict=False)
    missing = [k for k in missing if "position_ids" not in k]
    assert not missing and not unexpected, (missing, unexpected)
    # transformers' eager attention takes the softmax in float32; the fixture
    # keeps the whole forward in float64 (same math, softmax in the input dtype)
    import transformers.models.clip.modeling_clip as mc
    stock = mc.eager_attention_forward

    def attention_f64(module, query, key, value, attention_mask, scaling, dropout=0.0, **kw):
        w_ = torch.matmul(query, key.transpose(-1, -2)) * scaling
        if attention_mask is not None:
            w_ = w_ + attention_mask
        w_ = torch.softmax(w_, dim=-1)
        return torch.matmul(w_, value).transpose(1, 2).contiguous(), w_

    mc.eager_attention_forward = attention_f64
    try:
        with torch.no_grad():
            e = model(input_ids=torch.from_numpy(ids.astype(np.int64))).text_embeds.numpy()
    finally:
        mc.eager_attention_forward = stock
    return e / np.maximum(np.linalg.norm(e, axis=-1, keepdims=True), 1e-12)


def clip_text_fixture(name, cfg: ClipTextConfig, seed, lens, S):
    # std 0.1: the blocks move the residual stream well away from the embeddings
    w = random_clip_text_weights(cfg, seed, std=0.1)
    ids = random_clip_text_batch(len(lens), S, lens, seed + 1, cfg.vocab_size)
    embed = hf_clip_text_embed(w, cfg, ids)
    arrs = {"w::" + k: v for k, v in w.items()}
    arrs.update({"ids": ids, "embed": embed,
                 "config_json": np.frombuffer(json.dumps(cfg.to_open_clip_config()).encode(), dtype=np.uint8)})
    np.savez_compressed(os.path.join(HERE, name), **arrs)
    print("wrote", name, embed.shape)


def hf_modernbert_hidden(w: dict, cfg: dict, ids, mask) -> np.ndarray:
    """HF ``ModernBertModel`` in float64 with every layer global (the reference
    applies one global RoPE to all layers, modernbert.rs:64-71) and the
    reference's RoPE table (theta in float64, cos / sin stored as float32,
    modernbert.rs:106-131); transformers computes that table in float32 and
    takes RoPE and the softmax in float32, so those three steps are replaced by
    float64 ones here."""
    from transformers import ModernBertConfig, ModernBertModel
    import transformers.models.modernbert.modeling_modernbert as mm
    from oracle.bert import modernbert_rope_tables
    L = cfg["num_hidden_layers"]
    d = cfg["hidden_size"] // cfg["num_attention_heads"]
    hcfg = ModernBertConfig(vocab_size=cfg["vocab_size"], hidden_size=cfg["hidden_size"],
                            intermediate_size=cfg["intermediate_size"], num_hidden_layers=L,
                            num_attention_heads=cfg["num_attention_heads"], hidden_activation="gelu",
                            max_position_embeddings=cfg["max_position_embeddings"],
                            norm_eps=cfg.get("layer_norm_eps", 1e-5), norm_bias=False,
                            attention_bias=False, mlp_bias=False, pad_token_id=0,
                            global_rope_theta=cfg["global_rope_theta"])
    hcfg.layer_types = ["full_attention"] * L  # set after validation of the RoPE parameters
    hcfg._attn_implementation = "eager"
    model = ModernBertModel(hcfg).eval().to(torch.float64)
    sd = {k[len("model."):]: torch.from_numpy(np.asarray(v, dtype=np.float64)) for k, v in w.items()}
    missing, unexpected = model.load_state_dict(sd, strict=False)
    assert not missing and not unexpected, (missing, unexpected)
    cos_h, sin_h = modernbert_rope_tables(d, cfg["max_position_embeddings"], cfg["global_rope_theta"])

    def rotary_f64(self, x, position_ids, layer_type=None):
        pos = position_ids[0].numpy()
        c = np.concatenate([cos_h, cos_h], -1)[pos].astype(np.float64)
        s_ = np.concatenate([sin_h, sin_h], -1)[pos].astype(np.float64)
        return torch.from_numpy(c)[None], torch.from_numpy(s_)[None]

    def rope_f64(q, k, cos, sin, unsqueeze_dim=1):
        cos, sin = cos.unsqueeze(unsqueeze_dim), sin.unsqueeze(unsqueeze_dim)
        return q * cos + mm.rotate_half(q) * sin, k * cos + mm.rotate_half(k) * sin

    def attention_f64(module, query, key, value, attention_mask, scaling, dropout=0.0, **kw):
        a = torch.matmul(query, key.transpose(2, 3)) * scaling
        if attention_mask is not None:
            a = a + attention_mask
        a = torch.softmax(a, dim=-1)
        return torch.matmul(a, value).transpose(1, 2).contiguous(), a

    stock = (mm.ModernBertRotaryEmbedding.forward, mm.apply_rotary_pos_emb, mm.eager_attention_forward)
    mm.ModernBertRotaryEmbedding.forward = rotary_f64
    mm.apply_rotary_pos_emb, mm.eager_attention_forward = rope_f64, attention_f64
    try:
        with torch.no_grad():
            out = model(input_ids=torch.from_numpy(ids.astype(np.int64)),
                        attention_mask=torch.from_numpy(mask.astype(np.int64))).last_hidden_state
    finally:
        mm.ModernBertRotaryEmbedding.forward, mm.apply_rotary_pos_emb, mm.eager_attention_forward = stock
    return (out * torch.from_numpy(mask.astype(np.float64))[:, :, None]).numpy()


def modernbert_fixture(name, cfg: dict, seed, lens, S):
    from oracle.bert import random_modernbert_weights, random_token_batch
    w = random_modernbert_weights(cfg, seed, std=0.1)
    ids, mask = random_token_batch(len(lens), S, lens, seed + 1, id_lo=1,
                                   id_hi=cfg["vocab_size"] - 1, cls_id=1, sep_id=2)
    hidden = hf_modernbert_hidden(w, cfg, ids, mask)
    pooled = torch_pool_all(torch.from_numpy(hidden), torch.from_numpy(mask.astype(np.int64)))
    arrs = {"w::" + k: v for k, v in w.items()}
    arrs.update({"ids": ids, "mask": mask, "hidden": hidden,
                 "config_json": np.frombuffer(json.dumps(cfg).encode(), dtype=np.uint8)})
    arrs.update({"pooled_" + k: v.numpy() for k, v in pooled.items()})
    np.savez_compressed(os.path.join(HERE, name), **arrs)
    print("wrote", name, hidden.shape)


def reference_fixture():
    st = os.path.join(REF_TINY_BERT, "model.safetensors") if REF_TINY_BERT else ""
    if not st or not os.path.exists(st):
        print("reference checkout absent: reference_tiny_bert.npz not regenerated")
        return
    from safetensors.numpy import load_file
    w = load_file(st)
    cfg = BertConfig.from_dict(json.load(open(os.path.join(REF_TINY_BERT, "config.json"))))
    # the all-padding-row case of crates/jammi-encoders/tests/it/bert.rs:260-315
    # plus ragged rows (ids < vocab 256)
    ids = np.array([[1, 2, 3, 4, 5, 0, 0, 0], [0] * 8, [7, 9, 11, 0, 0, 0, 0, 0],
                    [101, 50, 60, 70, 80, 90, 100, 102]], dtype=np.uint32)
    mask = (np.arange(8)[None, :] < np.array([5, 0, 3, 8])[:, None]).astype(np.uint32)
    hidden = hf_bert_hidden(w, cfg, ids, mask)
    pooled = torch_pool_all(torch.from_numpy(hidden), torch.from_numpy(mask.astype(np.int64)))
    sha = hashlib.sha256(open(st, "rb").read()).hexdigest()
    arrs = {"ids": ids, "mask": mask, "hidden": hidden,
            "sha256": np.frombuffer(sha.encode(), dtype=np.uint8)}
    arrs.update({"pooled_" + k: v.numpy() for k, v in pooled.items()})
    np.savez_compressed(os.path.join(HERE, "reference_tiny_bert.npz"), **arrs)
    print("wrote reference_tiny_bert.npz sha256", sha)


def main():
    tiny = BertConfig(hidden_size=32, num_hidden_layers=1, num_attention_heads=2,
                      intermediate_size=128, vocab_size=256, max_position_embeddings=128)
    bert_fixture("tiny_bert_seeded.npz", tiny, seed=1234, lens=[16, 9, 1, 0, 13, 5], S=16)
    small = BertConfig(hidden_size=64, num_hidden_layers=2, num_attention_heads=4,
                       intermediate_size=256, vocab_size=512, max_position_embeddings=64)
    bert_fixture("small_bert_prefixed.npz", small, seed=99, lens=[40, 33, 64, 2, 17], S=64,
                 prefix="bert.")
    c = ClipVisionConfig(width=32, layers=1, heads=4, mlp_ratio=4.0, image_size=8,
                         patch_size=4, embed_dim=16, global_average_pool=True)
    clip_fixture("tiny_clip_gap.npz", c, seed=7, batch=3)
    c2 = ClipVisionConfig(width=32, layers=2, heads=4, mlp_ratio=4.0, image_size=8,
                          patch_size=4, embed_dim=16, global_average_pool=False)
    clip_fixture("tiny_clip_cls.npz", c2, seed=8, batch=3)
    distil = BertConfig(hidden_size=64, num_hidden_layers=2, num_attention_heads=4,
                        intermediate_size=256, vocab_size=512, max_position_embeddings=64)
    distilbert_fixture("small_distilbert.npz", distil, seed=321, lens=[64, 17, 1, 0, 40], S=64)
    ct = ClipTextConfig(width=64, layers=2, heads=4, context_length=24, vocab_size=300,
                        embed_dim=32)
    clip_text_fixture("small_clip_text.npz", ct, seed=505, lens=[24, 7, 2, 15, 24, 11], S=24)
    mb = {"model_type": "modernbert", "hidden_size": 64, "num_hidden_layers": 3,
          "num_attention_heads": 4, "intermediate_size": 96, "vocab_size": 300,
          "max_position_embeddings": 80, "layer_norm_eps": 1e-5, "global_rope_theta": 160000.0}
    modernbert_fixture("small_modernbert.npz", mb, seed=808, lens=[70, 33, 1, 0, 64, 9], S=70)
    reference_fixture()


if __name__ == "__main__":
    main()
