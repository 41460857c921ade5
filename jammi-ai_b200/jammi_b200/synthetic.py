"""Seeded synthetic weights and token batches for the benchmark workloads.

No dataset or checkpoint is involved: weights are random-init N(0, 0.02)
with LayerNorm gain 1 / bias 0 (the recipe of the reference's
tests/fixtures/generate_tiny_bert.py), token ids uniform in [1000, 30521]
with [CLS]=101 first and [SEP]=102 at each row's end, right padding.
"""
from __future__ import annotations

import numpy as np

BERT_BASE = dict(hidden_size=768, num_hidden_layers=12, num_attention_heads=12,
                 intermediate_size=3072, vocab_size=30522, max_position_embeddings=512,
                 type_vocab_size=2, layer_norm_eps=1e-12, model_type="bert")
BERT_LARGE = dict(BERT_BASE, hidden_size=1024, num_hidden_layers=24, num_attention_heads=16,
                  intermediate_size=4096)
MINILM_L6 = dict(BERT_BASE, hidden_size=384, num_hidden_layers=6, intermediate_size=1536)


def bert_weights(cfg: dict, seed: int, std: float = 0.02) -> dict:
    rng = np.random.default_rng(seed)
    H, F = cfg["hidden_size"], cfg["intermediate_size"]
    r = lambda *s: rng.standard_normal(s, dtype=np.float32) * np.float32(std)
    z = lambda n: np.zeros((n,), np.float32)
    o = lambda n: np.ones((n,), np.float32)
    w = {"embeddings.word_embeddings.weight": r(cfg["vocab_size"], H),
         "embeddings.position_embeddings.weight": r(cfg["max_position_embeddings"], H),
         "embeddings.token_type_embeddings.weight": r(cfg.get("type_vocab_size", 2), H),
         "embeddings.LayerNorm.weight": o(H), "embeddings.LayerNorm.bias": z(H)}
    for n in range(cfg["num_hidden_layers"]):
        p = f"encoder.layer.{n}."
        for nm in ("query", "key", "value"):
            w[p + f"attention.self.{nm}.weight"] = r(H, H)
            w[p + f"attention.self.{nm}.bias"] = z(H)
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


def uniform_lengths(rng, n: int, lo: int, hi: int) -> np.ndarray:
    return rng.integers(lo, hi + 1, size=n).astype(np.uint32)


def lognormal_lengths(rng, n: int, mu: float, sigma: float, lo: int, hi: int) -> np.ndarray:
    return np.clip(np.round(rng.lognormal(mu, sigma, size=n)), lo, hi).astype(np.uint32)


def token_batch(rng, lens, seq: int, id_lo: int = 1000, id_hi: int = 30521) -> np.ndarray:
    """Right-padded ids [len(lens), seq]; padding id 0."""
    B = len(lens)
    ids = rng.integers(id_lo, id_hi + 1, size=(B, seq), dtype=np.int64).astype(np.uint32)
    pos = np.arange(seq)[None, :]
    L = np.asarray(lens)[:, None]
    ids[pos >= L] = 0
    ids[:, 0] = np.where(np.asarray(lens) > 0, 101, 0)
    last = np.maximum(np.asarray(lens, dtype=np.int64) - 1, 0)
    rows = np.arange(B)
    ids[rows[np.asarray(lens) > 1], last[np.asarray(lens) > 1]] = 102
    return ids
