"""Pin the CPU oracle: the reference's known answers and the golden vectors."""
import hashlib
import json
import math
import os

import numpy as np
import pytest

from conftest import load_golden, reference_path
from oracle import bert as ob
from oracle import clip as oc
from oracle import image as oimg
from oracle import quant as oq

REF_FIXTURE = reference_path("cookbook", "fixtures", "tiny_bert")


# ── crates/jammi-encoders/tests/it/pooling.rs:15-83 (known answers) ─────────

def _hidden_fixture():
    return np.array([[[1.0, 0.0], [0.0, 1.0], [2.0, 2.0]]], dtype=np.float32)


def test_pooling_mean_ignores_padding():
    out = ob.pool_and_normalize(_hidden_fixture(), np.array([[1, 1, 0]]), ob.POOL_MEAN)[0]
    assert abs(out[0] - 1 / math.sqrt(2)) < 1e-6 and abs(out[1] - 1 / math.sqrt(2)) < 1e-6


def test_pooling_mean_all_real():
    out = ob.pool_and_normalize(_hidden_fixture(), np.array([[1, 1, 1]]), ob.POOL_MEAN)[0]
    assert abs(np.linalg.norm(out) - 1) < 1e-6 and abs(out[0] - out[1]) < 1e-6


def test_pooling_cls():
    out = ob.pool_and_normalize(_hidden_fixture(), np.array([[1, 1, 1]]), ob.POOL_CLS)[0]
    assert abs(out[0] - 1) < 1e-6 and abs(out[1]) < 1e-6


def test_pooling_max_excludes_padding():
    out = ob.pool_and_normalize(_hidden_fixture(), np.array([[1, 1, 0]]), ob.POOL_MAX)[0]
    assert abs(out[0] - 1 / math.sqrt(2)) < 1e-6 and abs(out[1] - 1 / math.sqrt(2)) < 1e-6


def test_pooling_weighted_mean():
    out = ob.pool_and_normalize(_hidden_fixture(), np.array([[1, 1, 1]]), ob.POOL_WEIGHTED_MEAN)[0]
    d = math.sqrt(113.0)
    assert abs(out[0] - 7 / d) < 1e-5 and abs(out[1] - 8 / d) < 1e-5


def test_pooling_all_padding_row_is_zero_or_finite():
    # tests/it/bert.rs:260-315: all-padding row -> exact zero for mean and
    # weighted-mean; finite for max.
    h = np.random.default_rng(0).standard_normal((2, 5, 8)).astype(np.float32)
    m = np.array([[1] * 5, [0] * 5])
    for s in (ob.POOL_MEAN, ob.POOL_WEIGHTED_MEAN, ob.POOL_MAX):
        out = ob.pool_and_normalize(h, m, s)
        assert np.all(np.isfinite(out))
        if s != ob.POOL_MAX:
            assert np.all(np.abs(out[1]) < 1e-6)
    # max: -1e30 sentinel, squared norm overflows f32, clamp at f32::MAX
    out = ob.pool_and_normalize(h, m, ob.POOL_MAX)[1]
    np.testing.assert_allclose(out, np.float32(-1e30) / np.finfo(np.float32).max, rtol=1e-6)


def test_extended_mask_values():
    ext = ob.extended_attention_mask(np.array([[1, 0, 1]], dtype=np.uint32))
    assert ext.shape == (1, 1, 1, 3)
    assert list(ext[0, 0, 0]) == [0.0, -10000.0, 0.0]


def test_sequence_too_long():
    cfg = ob.BertConfig(32, 1, 2, 128, 256, 8)
    w = ob.random_bert_weights(cfg, 0)
    with pytest.raises(ob.SequenceTooLong):
        ob.bert_forward_hidden(w, cfg, np.zeros((1, 9), np.uint32), np.ones((1, 9), np.uint32))


# ── golden vectors (HF transformers, float64) ───────────────────────────────

@pytest.mark.parametrize("name", ["tiny_bert_seeded.npz", "small_bert_prefixed.npz"])
def test_bert_oracle_matches_golden(name):
    w, g = load_golden(name)
    cfg = ob.BertConfig.from_dict(json.loads(bytes(g["config_json"]).decode()))
    valid = g["mask"].astype(bool)
    h64 = ob.bert_forward_hidden(w, cfg, g["ids"], g["mask"], dtype=np.float64)
    np.testing.assert_allclose(h64[valid], g["hidden"][valid], atol=1e-9, rtol=0)
    h32 = ob.bert_forward_hidden(w, cfg, g["ids"], g["mask"], dtype=np.float32)
    np.testing.assert_allclose(h32[valid], g["hidden"][valid], atol=2e-5, rtol=0)
    nonempty = g["mask"].sum(1) > 0
    for pname, pid in ob.POOLING_NAMES.items():
        out = ob.pool_and_normalize(h64, g["mask"], pid)
        # CLS of an all-padding row reads a padded position, whose hidden
        # state depends on the mask constant (-10000 in mask.rs:14-20, the
        # dtype minimum in transformers); every other strategy masks it out.
        rows = nonempty if pid == ob.POOL_CLS else slice(None)
        np.testing.assert_allclose(out[rows], g["pooled_" + pname][rows], atol=1e-9, rtol=0)


def test_distilbert_oracle_matches_golden():
    w, g = load_golden("small_distilbert.npz")
    d_cfg = json.loads(bytes(g["config_json"]).decode())
    valid = g["mask"].astype(bool)
    h64 = ob.distilbert_forward_hidden(w, d_cfg, g["ids"], g["mask"])
    np.testing.assert_allclose(h64[valid], g["hidden"][valid], atol=1e-9, rtol=0)
    nonempty = g["mask"].sum(1) > 0
    for pname, pid in ob.POOLING_NAMES.items():
        out = ob.pool_and_normalize(h64, g["mask"], pid)
        rows = nonempty if pid == ob.POOL_CLS else slice(None)
        np.testing.assert_allclose(out[rows], g["pooled_" + pname][rows], atol=1e-9, rtol=0)


def test_modernbert_oracle_matches_golden():
    """ModernBert::forward_hidden restated against HF ModernBertModel (f64,
    every layer global, the reference's RoPE table)."""
    w, g = load_golden("small_modernbert.npz")
    cfg = json.loads(bytes(g["config_json"]).decode())
    valid = g["mask"].astype(bool)
    h64 = ob.modernbert_forward_hidden(w, cfg, g["ids"], g["mask"])
    np.testing.assert_allclose(h64[valid], g["hidden"][valid], atol=1e-9, rtol=0)
    nonempty = g["mask"].sum(1) > 0
    for pname, pid in ob.POOLING_NAMES.items():
        out = ob.pool_and_normalize(h64, g["mask"], pid)
        rows = nonempty if pid == ob.POOL_CLS else slice(None)
        np.testing.assert_allclose(out[rows], g["pooled_" + pname][rows], atol=1e-9, rtol=0)


def test_modernbert_rope_table():
    """RotaryEmbedding::new (modernbert.rs:106-131): position 0 is the
    identity rotation; theta_i = pos * base^(-2i/d)."""
    c, s = ob.modernbert_rope_tables(8, 4, 10000.0)
    assert np.all(c[0] == 1) and np.all(s[0] == 0)
    assert abs(float(c[3, 1]) - math.cos(3 * 10000.0 ** (-2 / 8))) < 1e-7
    x = np.arange(8, dtype=np.float64)[None, None, None, :]
    np.testing.assert_array_equal(ob.rope_apply(x, c[:1], s[:1]), x)


def test_bert_oracle_on_reference_fixture():
    z = np.load(os.path.join(os.path.dirname(__file__), "golden", "reference_tiny_bert.npz"))
    st = os.path.join(REF_FIXTURE, "model.safetensors") if REF_FIXTURE else ""
    if not st or not os.path.exists(st):
        pytest.skip("reference checkout not present")
    assert hashlib.sha256(open(st, "rb").read()).hexdigest() == bytes(z["sha256"]).decode()
    from safetensors.numpy import load_file
    w = load_file(st)
    cfg = ob.BertConfig.from_dict(json.load(open(os.path.join(REF_FIXTURE, "config.json"))))
    h = ob.bert_forward_hidden(w, cfg, z["ids"], z["mask"])
    valid = z["mask"].astype(bool)
    np.testing.assert_allclose(h[valid], z["hidden"][valid], atol=1e-9, rtol=0)
    nonempty = z["mask"].sum(1) > 0
    for pname, pid in ob.POOLING_NAMES.items():
        rows = nonempty if pid == ob.POOL_CLS else slice(None)
        np.testing.assert_allclose(ob.pool_and_normalize(h, z["mask"], pid)[rows],
                                   z["pooled_" + pname][rows], atol=1e-9)
    # all-padding row (row 1) -> exact zero vector for mean pooling
    assert np.all(ob.pool_and_normalize(h, z["mask"], ob.POOL_MEAN)[1] == 0)


@pytest.mark.parametrize("name", ["tiny_clip_gap.npz", "tiny_clip_cls.npz"])
def test_clip_oracle_matches_golden(name):
    w, g = load_golden(name)
    cfg = oc.ClipVisionConfig.from_open_clip_config(json.loads(bytes(g["config_json"]).decode()))
    raw = oc.clip_vision_forward(w, cfg, g["pixels"])
    np.testing.assert_allclose(raw, g["embed_raw"], atol=1e-9, rtol=0)
    np.testing.assert_allclose(oc.l2_normalize_image(raw), g["embed"], atol=1e-9, rtol=0)


def test_clip_text_oracle_matches_golden():
    """ClipText::forward restated against HF CLIPTextModelWithProjection (f64)."""
    w, g = load_golden("small_clip_text.npz")
    cfg = oc.ClipTextConfig.from_open_clip_config(json.loads(bytes(g["config_json"]).decode()))
    e = oc.clip_text_forward(w, cfg, g["ids"])
    np.testing.assert_allclose(e, g["embed"], atol=1e-9, rtol=0)
    np.testing.assert_allclose(np.linalg.norm(e, axis=1), 1.0, atol=1e-12)


def test_clip_text_oracle_causal_and_eot():
    """Under the causal mask, ids after the EOT token (the row's largest id)
    cannot reach the pooled position (clip_text.rs:287-295, 322-326); a longer
    context than the config's is SequenceTooLong (:302-308)."""
    w, g = load_golden("small_clip_text.npz")
    cfg = oc.ClipTextConfig.from_open_clip_config(json.loads(bytes(g["config_json"]).decode()))
    ids = g["ids"].copy()
    eot = ids.argmax(1)
    rng = np.random.default_rng(1)
    for b in range(ids.shape[0]):
        tail = ids.shape[1] - eot[b] - 1
        ids[b, eot[b] + 1:] = rng.integers(1, cfg.vocab_size - 2, size=tail)
    np.testing.assert_allclose(oc.clip_text_forward(w, cfg, ids), g["embed"], atol=1e-12, rtol=0)
    with pytest.raises(ValueError):
        oc.clip_text_forward(w, cfg, np.zeros((1, cfg.context_length + 1), np.uint32))


# ── int8 format: integer-exact properties ───────────────────────────────────

def test_quantize_rows_properties():
    rng = np.random.default_rng(3)
    x = rng.standard_normal((64, 96)).astype(np.float32) * rng.uniform(0.01, 10, size=(64, 1)).astype(np.float32)
    x[5] = 0.0
    q, s = oq.quantize_rows(x)
    assert q.dtype == np.int8 and np.abs(q.astype(int)).max() <= 127
    # the element of largest magnitude maps to +-127 in every non-zero row
    nz = np.abs(x).max(1) > 0
    assert np.all(np.abs(q[nz]).max(1) == 127)
    assert np.all(q[5] == 0) and s[5] == 0
    # dequantised error is at most half a step
    err = np.abs(q.astype(np.float64) * s[:, None] - x)
    assert np.all(err <= 0.5 * s[:, None] * (1 + 1e-6) + 1e-30)


def test_gemm_s8_s32_exact():
    rng = np.random.default_rng(4)
    a = rng.integers(-127, 128, size=(33, 4096), dtype=np.int64).astype(np.int8)
    b = rng.integers(-127, 128, size=(17, 4096), dtype=np.int64).astype(np.int8)
    a[0, :] = 127; b[0, :] = 127  # the largest possible accumulator at K=4096
    acc = oq.gemm_s8_s32(a, b)
    assert acc[0, 0] == 4096 * 127 * 127
    ref = np.array([[int(np.dot(a[i].astype(object), b[j].astype(object))) for j in range(3)] for i in range(3)])
    assert np.array_equal(acc[:3, :3], ref)


def test_int8_bert_close_to_float():
    cfg = ob.BertConfig(64, 2, 4, 256, 512, 64)
    w = ob.random_bert_weights(cfg, 11)
    ids, mask = ob.random_token_batch(4, 32, [32, 20, 7, 1], seed=5, id_lo=1, id_hi=511, cls_id=1, sep_id=2)
    ref = ob.pool_and_normalize(ob.bert_forward_hidden(w, cfg, ids, mask), mask)
    q = ob.pool_and_normalize(oq.bert_int8_forward_hidden(w, cfg, ids, mask), mask)
    cos = (ref * q).sum(1)
    assert np.all(cos > 0.999), cos


# ── int8 format with bf16 storage between operators ─────────────────────────

def test_bf16_round_matches_torch():
    torch = pytest.importorskip("torch")
    rng = np.random.default_rng(31)
    x = (rng.standard_normal(200000) * np.exp(rng.uniform(-20, 20, 200000))).astype(np.float32)
    # ties: values exactly halfway between two bf16 neighbours, both parities
    x[:4] = np.array([1.0 + 2.0**-8, 1.0 + 3 * 2.0**-8, -(1.0 + 2.0**-8), 0.0], dtype=np.float32)
    ref = torch.from_numpy(x).to(torch.bfloat16).float().numpy()
    got = oq.bf16_round(x.astype(np.float64))
    assert got.dtype == np.float32 and np.array_equal(got, ref)
    assert got[0] == 1.0 and got[1] == 1.0 + 2.0**-6 and got[2] == -1.0
    assert np.array_equal(oq.bf16_round_f32(x), ref)


def test_gemm_s8_exact_at_the_extremes():
    """Float32 BLAS over 1024-wide K chunks is exact even at |acc| = 4096 * 128^2."""
    rng = np.random.default_rng(32)
    a = rng.integers(-128, 128, size=(9, 4096), dtype=np.int64).astype(np.int8)
    b = rng.integers(-128, 128, size=(7, 4096), dtype=np.int64).astype(np.int8)
    a[0, :] = -128; b[0, :] = -128; a[1, :] = 127; b[1, :] = -128
    acc = oq.gemm_s8_exact(a, b)
    assert acc[0, 0] == 4096 * 128 * 128 and acc[1, 1] == -4096 * 127 * 128
    assert np.array_equal(acc, a.astype(np.int64) @ b.astype(np.int64).T)
    assert np.array_equal(oq.gemm_s8_exact(a[:, :1024], b[:, :1024]),
                          a[:, :1024].astype(np.int64) @ b[:, :1024].astype(np.int64).T)


def test_dequant_f32_is_one_fma_then_the_residual():
    acc = np.array([[16777217, -3]], dtype=np.int64)          # 2^24 + 1 rounds to 2^24 in f32
    s_tok = np.array([0.5], np.float32)
    s_ch = np.array([2.0, np.float32(1.0 / 3.0)], np.float32)
    bias = np.array([4.0, 0.25], np.float32)
    y = oq.dequant_f32(acc, s_tok, s_ch, bias, resid=np.array([[2.0, 1.0]], np.float32))
    assert y[0, 0] == 16777216.0 + 4.0 + 2.0                 # not 2^24 + 1 + 4 + 2
    s1 = np.float32(np.float32(0.5) * np.float32(1.0 / 3.0))
    want = np.float32(np.float32(-3.0 * np.float64(s1) + 0.25) + np.float32(1.0))
    assert y[0, 1] == want
    # a zero bias takes the float32 product, which is the same single rounding
    y0 = oq.dequant_f32(acc, s_tok, s_ch, np.zeros(2, np.float32))
    assert y0[0, 1] == np.float32(-3.0 * np.float64(s1))


def test_int8_bf16_oracle_agrees_with_float64_int8_oracle():
    """The two int8 restatements differ only by the bf16 storage of the
    activations: a few int8 codes at rounding boundaries."""
    cfg = ob.BertConfig(64, 2, 4, 256, 512, 64)
    w = ob.random_bert_weights(cfg, 11)
    lens = np.array([32, 20, 7, 1, 0])
    ids, mask = ob.random_token_batch(5, 32, lens, seed=5, id_lo=1, id_hi=511, cls_id=1, sep_id=2)
    f64 = ob.pool_and_normalize(oq.bert_int8_forward_hidden(w, cfg, ids, mask), mask)
    b16 = oq.bert_int8_bf16_embed(w, cfg, ids, lens)
    cos = (f64[:4] * b16[:4]).sum(1)
    assert np.all(cos > 0.999), cos
    assert np.all(b16[4] == 0)                                # empty row -> zero vector
    h, cu = oq.bert_int8_bf16_forward(w, cfg, ids, lens)
    assert h.shape == (int(lens.sum()), 64) and list(cu) == [0, 32, 52, 59, 60, 60]
    assert h.dtype == np.float32 and np.array_equal(oq.bf16_round_f32(h), h)   # all bf16 values


def test_attention_bf16_p_is_the_softmax_up_to_bf16_p():
    """The device's P V emulation differs from the exact softmax only by P's
    bf16 rounding, for every block structure; with one block and no rescale
    it equals P = bf16(2^(t - max)) / sum(2^(t - max)) exactly."""
    rng = np.random.default_rng(33)
    q, k, v = (rng.standard_normal((n, 64)) for n in (40, 300, 300))
    k[130:140] *= 8.0                                  # a later block dominates
    exact = ob.softmax_last(q @ k.T / 8.0) @ v
    for block, thr in (oq.ATTN_TC, oq.ATTN_MMA, (300, 8.0)):
        got = oq.attention_bf16_p(q, k, v, 1 / 8.0, block, thr)
        assert np.abs(got - exact).max() < 2e-2 * np.abs(v).max()
    t = q @ k.T / 8.0 * oq.LOG2E
    p = np.exp2(t - t.max(1, keepdims=True))
    want = (oq.bf16_round(p).astype(np.float64) @ v) / p.sum(1, keepdims=True)
    np.testing.assert_allclose(oq.attention_bf16_p(q, k, v, 1 / 8.0, 300, 8.0), want, rtol=1e-12)


def test_projection_head_oracle():
    """LoraLinear over an identity base: x + (alpha/rank) (x A^T) B^T; a zero B
    leaves the embedding unchanged (LoRA's standard init, lora_linear.rs)."""
    x = np.array([[0.6, 0.8, 0.0], [1.0, 0.0, 0.0]])
    a = np.array([[1.0, 0.0, 0.0], [0.0, 1.0, 0.0]])   # rank 2
    b = np.array([[0.0, 1.0], [1.0, 0.0], [0.5, 0.5]])
    y = ob.projection_head(x, a, b, lora_alpha=4.0)       # scaling 2
    # x A^T = [[0.6, 0.8], [1, 0]]; (x A^T) B^T = [[0.8, 0.6, 0.7], [0, 1, 0.5]]
    assert np.allclose(y, [[0.6 + 1.6, 0.8 + 1.2, 1.4], [1.0, 2.0, 1.0]])
    assert np.array_equal(ob.projection_head(x, a, np.zeros_like(b), 8.0), x)


# ── image preprocessing (image_preprocess.rs) ────────────────────────────────

def test_pad_to_square_known_answers():
    """image_preprocess.rs:95-119: landscape, portrait and square shapes."""
    assert oimg.pad_to_square(np.zeros((100, 200, 3), np.uint8)).shape == (200, 200, 3)
    assert oimg.pad_to_square(np.zeros((300, 100, 3), np.uint8)).shape == (300, 300, 3)
    sq = np.zeros((150, 150, 3), np.uint8)
    assert oimg.pad_to_square(sq) is sq
    # centred on white: (size - w) / 2 columns of 255 on the left
    p = oimg.pad_to_square(np.zeros((2, 5, 3), np.uint8))
    assert np.all(p[0] == 255) and np.all(p[1:3] == 0) and np.all(p[3:] == 255)


def test_preprocess_known_answers():
    """image_preprocess.rs:121-146: batch shape, and a white image maps to
    (1 - mean) / std in every pixel of channel 0."""
    out = oimg.preprocess_image_batch([np.zeros((200, 100, 3), np.uint8),
                                       np.zeros((150, 300, 3), np.uint8)], 224)
    assert out.shape == (2, 3, 224, 224)
    white = np.full((10, 10, 3), 255, np.uint8)
    v = oimg.preprocess_image_batch([white], 4)
    exp = (np.float32(1.0) - np.float32(oimg.OPENAI_CLIP_MEAN[0])) / np.float32(oimg.OPENAI_CLIP_STD[0])
    assert np.all(v[0, 0] == exp)
    with pytest.raises(ValueError):
        oimg.preprocess_image_batch([], 224)


def test_catmull_rom_resize_properties():
    """Catmull-Rom interpolates (k(0) = 1, k(+-1) = k(+-2) = 0), so a same-size
    resize is the identity; weights form a partition of unity; a constant
    image stays constant."""
    assert oimg.catmull_rom(0.0) == 1 and oimg.catmull_rom(1.0) == 0 and oimg.catmull_rom(-2.0) == 0
    img = oimg.random_images(3, [(37, 37)])[0]
    assert np.array_equal(oimg.resize_catmull_rom(img, 37), img)
    for o in (0, 17, 223):
        _, ws = oimg.taps(o, 1000, 224)
        assert abs(float(sum(ws)) - 1.0) < 1e-5
    flat = np.full((90, 90, 3), 77, np.uint8)
    assert np.all(oimg.resize_catmull_rom(flat, 224) == 77)
    assert np.all(oimg.resize_catmull_rom(flat, 20) == 77)
