"""End-to-end GPU parity of the encoder forward (through the C ABI) against
the golden vectors and the CPU oracle.

Acceptance (per row, on the L2-normalised embedding):
* f32 format:  max |gpu - ref| <= 1e-4 and cosine >= 0.9999
* bf16 format: max |gpu - ref| <= 2e-3 and cosine >= 0.9999
* int8 format: the same bf16 bar, against the int8 oracle with bf16 storage
  between operators (``oracle.quant.bert_int8_bf16_embed``: the same
  quantisation points and the same bf16 rounding points, integer-exact
  accumulation), on every row length; the s32 accumulators themselves are
  checked bit-exact in test_gpu_ops.py.
"""
import json

import numpy as np
import pytest

from conftest import load_golden
from oracle import bert as ob
from oracle import clip as oc
from oracle import quant as oq

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

# f16: the reference's own CPU <-> GPU acceptance bar (max |diff| <= 1e-3,
# crates/jammi-ai/tests/gpu_capability/harness.rs:40); f16 keeps 3 more
# mantissa bits than bf16.
TOL = {"f32": 1e-4, "bf16": 2e-3, "int8": 2e-3, "f16": 1e-3}
COS = 0.9999


@pytest.fixture(scope="module", autouse=True)
def _need_gpu():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def assert_close_rows(got, ref, fmt, rows=None, cos_bar=None):
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    if rows is not None:
        got, ref = got[rows], ref[rows]
    err = np.abs(got - ref).max(axis=1)
    nz = (np.linalg.norm(ref, axis=1) > 0.5)
    cos = (got * ref).sum(1)[nz] / (np.linalg.norm(got, axis=1)[nz] * np.linalg.norm(ref, axis=1)[nz])
    # The bars are stated for 768-wide embeddings (element RMS 1/sqrt(768)).
    # A unit vector of width D < 768 has elements sqrt(768/D) larger, and a
    # 16-bit format's error is relative, so the max-abs bar scales with it
    # for the small golden fixtures (D = 16..64); f32 keeps its absolute bar.
    D = got.shape[1]
    tol = TOL[fmt] * (max(1.0, (768.0 / D) ** 0.5) if fmt != "f32" else 1.0)
    print(f"{fmt} D={D}: max-abs {err.max():.3e} (bar {tol:.1e}), "
          f"min cos {cos.min() if cos.size else 1.0:.7f}")
    bar = COS if cos_bar is None else cos_bar
    assert err.max() <= tol, f"max-abs {err.max():.3e} > {tol:.2e} ({fmt})"
    assert cos.size == 0 or cos.min() >= bar, f"cosine {cos.min():.6f} < {bar} ({fmt})"
    return err.max(), (cos.min() if cos.size else 1.0)


def _bert(weights, cfg, fmt, pooling="mean"):
    from jammi_b200 import Bert
    return Bert.from_weights(weights, cfg, device=0, fmt=fmt, pooling=pooling)


# ── golden fixtures (HF transformers) ───────────────────────────────────────

@pytest.mark.parametrize("name", ["tiny_bert_seeded.npz", "small_bert_prefixed.npz"])
@pytest.mark.parametrize("fmt", ["f32", "bf16", "f16"])
def test_bert_golden_all_poolings(name, fmt):
    w, g = load_golden(name)
    cfg = json.loads(bytes(g["config_json"]).decode())
    model = _bert(w, cfg, fmt)
    lens = g["mask"].sum(1)
    for pname in ("mean", "cls", "max", "weighted_mean"):
        out = model.encode(g["ids"], lens, pooling=pname)
        rows = lens > 0 if pname == "cls" else None
        assert_close_rows(out, g["pooled_" + pname], fmt, rows)
    # all-padding row -> exact zero vector for mean pooling (tests/it/bert.rs:260-315)
    out = model.encode(g["ids"], lens, pooling="mean")
    assert np.all(out[lens == 0] == 0)


@pytest.mark.parametrize("fmt", ["f32", "bf16", "int8", "f16"])
def test_distilbert_golden(fmt):
    """DistilBERT weights and config (distilbert.rs) through the same forward,
    against HF DistilBertModel (f32 / bf16) or the int8 oracle."""
    from jammi_b200 import Bert
    from jammi_b200._lib import TEXT_DISTILBERT
    w, g = load_golden("small_distilbert.npz")
    d_cfg = json.loads(bytes(g["config_json"]).decode())
    ids, mask = g["ids"], g["mask"]
    lens = mask.sum(1)
    model = Bert.from_weights(w, d_cfg, device=0, fmt=fmt, pooling="mean")
    assert model.info.variant == TEXT_DISTILBERT
    out = model.encode(ids, lens)
    if fmt == "int8":  # the int8 oracle over the same weights, renamed onto BERT
        bw, cfg = ob.distilbert_as_bert(w, d_cfg)
        ref = oq.bert_int8_bf16_embed(bw, cfg, ids, lens)
    else:
        ref = g["pooled_mean"]
    assert_close_rows(out, ref, fmt)


def test_bert_forward_hidden_golden():
    w, g = load_golden("tiny_bert_seeded.npz")
    cfg = json.loads(bytes(g["config_json"]).decode())
    model = _bert(w, cfg, "f32")
    h = model.forward_hidden(g["ids"], g["mask"]).cpu().numpy()
    valid = g["mask"].astype(bool)
    assert np.abs(h[valid] - g["hidden"][valid]).max() <= 1e-4
    assert np.all(h[~valid] == 0)


def test_bert_forward_mask_api_matches_lengths():
    w, g = load_golden("tiny_bert_seeded.npz")
    cfg = json.loads(bytes(g["config_json"]).decode())
    model = _bert(w, cfg, "bf16")
    a = model.forward(g["ids"], g["mask"])
    b = model.encode(g["ids"], g["mask"].sum(1))
    assert np.array_equal(a, b)


@pytest.mark.parametrize("name", ["tiny_clip_gap.npz", "tiny_clip_cls.npz"])
@pytest.mark.parametrize("fmt", ["f32", "bf16"])
def test_clip_golden(name, fmt):
    from jammi_b200 import OpenClipVisionTransformer
    w, g = load_golden(name)
    cfg = json.loads(bytes(g["config_json"]).decode())
    model = OpenClipVisionTransformer.from_weights(w, cfg, device=0, fmt=fmt)
    out = model.forward_image(g["pixels"])
    assert_close_rows(out, g["embed"], fmt)


# ── benchmark-config shapes against the oracle ──────────────────────────────

def test_minilm_l6_f32_config():
    """MiniLM-L6 architecture, f32, batch 32 x seq 128, lengths U[16,128]."""
    cfg = ob.BertConfig(384, 6, 12, 1536, 30522, 512)
    w = ob.random_bert_weights(cfg, seed=101)
    rng = np.random.default_rng(102)
    lens = rng.integers(16, 129, size=32)
    ids, mask = ob.random_token_batch(32, 128, lens, seed=103)
    ref = ob.bert_forward(w, cfg, ids, mask)
    out = _bert(w, cfg.to_dict(), "f32").encode(ids, lens)
    assert_close_rows(out, ref, "f32")


def _bert_base(seed):
    cfg = ob.BertConfig(768, 12, 12, 3072, 30522, 512)
    return cfg, ob.random_bert_weights(cfg, seed=seed)


@pytest.mark.parametrize("tc_attention", [False, True])
def test_bert_base_bf16_config(tc_attention):
    """BERT-base, bf16, seq 256, lengths U[32,256] (batch reduced for the oracle),
    with the tcgen05 attention kernel (the default) and with the mma.sync one."""
    from jammi_b200 import ops
    cfg, w = _bert_base(201)
    rng = np.random.default_rng(202)
    lens = rng.integers(32, 257, size=12)
    lens[0] = 256
    ids, mask = ob.random_token_batch(12, 256, lens, seed=203)
    ref = ob.bert_forward(w, cfg, ids, mask)
    ops.set_attention_tcgen05(tc_attention)
    try:
        out = _bert(w, cfg.to_dict(), "bf16").encode(ids, lens)
    finally:
        ops.set_attention_tcgen05(True)
    assert_close_rows(out, ref, "bf16")


def test_bert_base_f16_config():
    """BERT-base in f16 (ComputePrecision::F16, crates/jammi-numerics/src/precision.rs:36-51):
    f16 weights and activations, f32 accumulation, seq 256, lengths U[32,256]."""
    cfg, w = _bert_base(211)
    rng = np.random.default_rng(212)
    lens = rng.integers(32, 257, size=12)
    lens[0] = 256
    ids, mask = ob.random_token_batch(12, 256, lens, seed=213)
    ref = ob.bert_forward(w, cfg, ids, mask)
    model = _bert(w, cfg.to_dict(), "f16")
    assert model.info.format == 3
    assert_close_rows(model.encode(ids, lens), ref, "f16")


def test_f16_is_defined_for_bert_and_distilbert_only(tmp_path):
    """f16 answers JB_ERR_INVALID for the families without an f16 path
    (ModernBERT, the OpenCLIP towers) and for LoRA adapters."""
    from jammi_b200 import JbError, OpenClipVisionTransformer
    w, g = load_golden("small_modernbert.npz")
    mcfg = json.loads(bytes(g["config_json"]).decode())
    with pytest.raises(JbError):
        _bert(w, mcfg, "f16")
    ccfg = oc.ClipVisionConfig(image_size=64, patch_size=32, width=64, layers=1, heads=2, embed_dim=32)
    with pytest.raises(JbError):
        OpenClipVisionTransformer.from_weights(oc.random_clip_weights(ccfg, seed=1),
                                               ccfg.to_open_clip_config(), device=0, fmt="f16")
    bw, bg = load_golden("tiny_bert_seeded.npz")
    bcfg = json.loads(bytes(bg["config_json"]).decode())
    model = _bert(bw, bcfg, "f16")
    H = bcfg["hidden_size"]
    with pytest.raises(JbError):
        model.set_lora(0, 0, np.zeros((8, H), np.float32), np.zeros((H, 8), np.float32), 1.0)


def test_bert_base_int8_config():
    """BERT-base with int8 weights (per-channel) and per-token int8 activations."""
    cfg, w = _bert_base(301)
    rng = np.random.default_rng(302)
    lens = rng.integers(32, 257, size=8)
    ids, mask = ob.random_token_batch(8, 256, lens, seed=303)
    ref = oq.bert_int8_bf16_embed(w, cfg, ids, lens)
    out = _bert(w, cfg.to_dict(), "int8").encode(ids, lens)
    assert_close_rows(out, ref, "int8")
    # and the quantisation error itself stays small against the float model
    fref = ob.bert_forward(w, cfg, ids, mask)
    assert (out * fref).sum(1).min() > 0.995


def test_bert_base_int8_sharded_job_lengths():
    """The sharded job's rows: BERT-base int8, 128 rows with lengths
    lognormal(4.5, 0.8) clipped to [8, 512] (about half of them under 96
    tokens), plus rows of exactly 8 tokens and one of 512, at the bar on
    every row."""
    cfg, w = _bert_base(501)
    rng = np.random.default_rng(502)
    lens = np.clip(np.round(rng.lognormal(4.5, 0.8, size=128)), 8, 512).astype(int)
    lens[:3] = (8, 8, 512)
    ids, _ = ob.random_token_batch(128, 512, lens, seed=503)
    ref = oq.bert_int8_bf16_embed(w, cfg, ids, lens)
    out = _bert(w, cfg.to_dict(), "int8").encode(ids, lens)
    assert_close_rows(out, ref, "int8")


def test_bert_base_int8_short_rows():
    """Rows of 1 to 48 tokens (a lone [CLS], [CLS] [SEP], ...): the mean pool
    averages little of the quantisation noise here, so these rows are the
    hardest for the int8 bar."""
    cfg, w = _bert_base(511)
    lens = np.arange(1, 49)
    ids, _ = ob.random_token_batch(48, 48, lens, seed=512)
    ref = oq.bert_int8_bf16_embed(w, cfg, ids, lens)
    out = _bert(w, cfg.to_dict(), "int8").encode(ids, lens)
    assert_close_rows(out, ref, "int8")


def _layer_norm_f32(x, g, b, eps):
    """LayerNorm evaluated in float32: a perturbation of the oracle at the
    level of f32 rounding, to measure how far such rounding moves the int8
    forward."""
    x = np.asarray(x, np.float32)
    g = np.asarray(g, np.float32)
    b = np.asarray(b, np.float32)
    m = x.mean(-1, keepdims=True, dtype=np.float32)
    c = x - m
    v = (c * c).mean(-1, keepdims=True, dtype=np.float32)
    return (c / np.sqrt(v + np.float32(eps)) * g + b).astype(np.float64)


def test_bert_large_prequantised_int8(monkeypatch):
    """BERT-large in the int8 checkpoint format, full depth (24 layers): int8
    weights with per-output-channel scales log-uniform in [1e-3, 1e-1];
    32 rows with lengths lognormal(5.0, 0.6) clipped to [8, 512].

    At this depth the int8 forward amplifies f32-rounding-level differences:
    each layer re-quantises its activations, so a rare bf16 flip upstream
    becomes a whole int8 step downstream.  The test measures that on the
    oracle itself -- the same oracle with its LayerNorm evaluated in float32
    instead of float64 -- and holds the device to the 2e-3 max-abs bar and
    to a cosine no further from 1 than twice the oracle's own spread (and at
    least 0.9998)."""
    cfg = ob.BertConfig(1024, 24, 16, 4096, 30522, 512)
    w = ob.random_bert_weights(cfg, seed=401)
    rng = np.random.default_rng(402)
    for n in range(cfg.num_hidden_layers):
        for lin, (o, i) in zip(oq.LINEARS, [(1024, 1024)] * 4 + [(4096, 1024), (1024, 4096)]):
            q, s = oq.random_int8_linear(o, i, rng)
            k = f"encoder.layer.{n}.{lin}"
            del w[k + ".weight"]
            w[k + ".weight_q"] = q
            w[k + ".weight_scale"] = s
    lens = np.clip(np.round(rng.lognormal(5.0, 0.6, size=32)), 8, 512).astype(int)
    lens[0] = 8
    ids, _ = ob.random_token_batch(32, int(lens.max()), lens, seed=403)
    ref = oq.bert_int8_bf16_embed(w, cfg, ids, lens)
    out = _bert(w, cfg.to_dict(), "int8").encode(ids, lens)
    err, cos = assert_close_rows(out, ref, "int8", cos_bar=0.9998)
    monkeypatch.setattr(oq, "layer_norm", _layer_norm_f32)
    ref32 = oq.bert_int8_bf16_embed(w, cfg, ids[:8], lens[:8])
    spread = 1.0 - float((ref[:8] * ref32).sum(1).min())
    print(f"oracle spread (LayerNorm f32 vs f64, 8 rows): 1 - cos = {spread:.2e}; "
          f"device: 1 - cos = {1.0 - cos:.2e}")
    assert 1.0 - cos <= max(2.0 * spread, 1e-4)


def test_clip_vit_b32_bf16_config():
    """CLIP ViT-B/32 vision tower, bf16, pixels N(0,1) (batch reduced for the oracle)."""
    from jammi_b200 import OpenClipVisionTransformer
    cfg = oc.ClipVisionConfig()
    w = oc.random_clip_weights(cfg, seed=501)
    px = np.random.default_rng(502).standard_normal((16, 3, 224, 224)).astype(np.float32)
    ref = oc.l2_normalize_image(oc.clip_vision_forward(w, cfg, px))
    model = OpenClipVisionTransformer.from_weights(w, cfg.to_open_clip_config(), device=0, fmt="bf16")
    assert_close_rows(model.forward_image(px), ref, "bf16")


# ── API behaviour ───────────────────────────────────────────────────────────

def test_host_and_device_entry_points_agree():
    cfg, w = _bert_base(601)
    rng = np.random.default_rng(602)
    lens = rng.integers(1, 129, size=40)
    ids, _ = ob.random_token_batch(40, 128, lens, seed=603)
    model = _bert(w, cfg.to_dict(), "bf16")
    host = model.encode(ids, lens)
    d_ids = torch.from_numpy(ids.astype(np.int32)).cuda()
    d_lens = torch.from_numpy(lens.astype(np.int32)).cuda()
    out = torch.empty((40, 768), device="cuda")
    model.encode_device(d_ids, d_lens, out, stream=torch.cuda.current_stream())
    model.sync(torch.cuda.current_stream())
    assert np.array_equal(out.cpu().numpy(), host)
    assert np.array_equal(model.encode(ids, lens), host)  # deterministic


def test_image_chunked_copy_matches_device_entry_point():
    """jb_encode_image copies a batch of more than 128 images in chunks, each
    chunk's forward overlapping the next chunk's copy: every row equals the
    whole-batch forward of jb_encode_image_device bit for bit, on the eager
    first call, the capturing second call and a replaying third call."""
    from jammi_b200 import OpenClipVisionTransformer
    cfg = oc.ClipVisionConfig()
    w = oc.random_clip_weights(cfg, seed=511)
    model = OpenClipVisionTransformer.from_weights(w, cfg.to_open_clip_config(), device=0, fmt="bf16")
    px = np.random.default_rng(512).standard_normal((300, 3, 224, 224)).astype(np.float32)
    d_px = torch.from_numpy(px).cuda()
    ref = torch.empty((300, model.info.output_dim), device="cuda")
    model.forward_image_device(d_px, ref, stream=torch.cuda.current_stream())
    model.sync(torch.cuda.current_stream())
    ref = ref.cpu().numpy()
    for _ in range(3):
        assert np.array_equal(model.forward_image(px), ref)
    # a batch of one chunk after the chunked ones (and the reverse order of sizes)
    assert np.array_equal(model.forward_image(px[:100]), ref[:100])
    assert np.array_equal(model.forward_image(px[:257]), ref[:257])
    model.close()


def test_sequence_too_long():
    from jammi_b200 import SequenceTooLong
    w, g = load_golden("tiny_bert_seeded.npz")
    cfg = json.loads(bytes(g["config_json"]).decode())
    model = _bert(w, cfg, "bf16")
    ids = np.ones((1, 129), np.uint32)
    with pytest.raises(SequenceTooLong):
        model.encode(ids, np.array([129], np.uint32))


def test_invalid_token_id_is_an_error():
    from jammi_b200 import JbError
    w, g = load_golden("tiny_bert_seeded.npz")
    cfg = json.loads(bytes(g["config_json"]).decode())
    model = _bert(w, cfg, "bf16")
    ids = np.full((2, 4), 7, np.uint32)
    ids[1, 2] = 256  # vocab is 256
    with pytest.raises(JbError):
        model.encode(ids, np.array([4, 4], np.uint32))
    # the handle stays usable afterwards
    ids[1, 2] = 5
    assert np.all(np.isfinite(model.encode(ids, np.array([4, 4], np.uint32))))


def test_graph_replay_matches_direct_launches():
    """The first call of a shape runs launch by launch, the second captures the
    forward as a CUDA graph and later calls replay it: outputs of replays with
    changing inputs equal the launch-by-launch results bit for bit, also for
    int8 and on the legacy default stream."""
    cfg, w = _bert_base(611)
    rng = np.random.default_rng(612)
    batches = []
    for k in range(2):
        lens = rng.integers(1, 97, size=24)
        ids, _ = ob.random_token_batch(24, 96, lens, seed=613 + k)
        batches.append((ids, lens))
    for fmt in ("bf16", "int8"):
        direct = [_bert(w, cfg.to_dict(), fmt).encode(ids, lens) for ids, lens in batches]
        model = _bert(w, cfg.to_dict(), fmt)
        for rep in range(3):  # direct, capture, replay, replay, ...
            for (ids, lens), ref in zip(batches, direct):
                assert np.array_equal(model.encode(ids, lens), ref), (fmt, rep)
        d_out = torch.empty((24, 768), device="cuda")
        for (ids, lens), ref in zip(batches, direct):
            model.encode_device(torch.from_numpy(ids.astype(np.int32)).cuda(),
                                torch.from_numpy(lens.astype(np.int32)).cuda(), d_out, stream=None)
            model.sync(None)
            assert np.array_equal(d_out.cpu().numpy(), ref), fmt


def test_graphs_follow_workspace_growth():
    """Captured graphs hold workspace pointers: a larger batch regrows the
    workspace, which must drop them; the original shape then re-runs (and
    re-captures) against the new buffers with unchanged results."""
    cfg, w = _bert_base(621)
    rng = np.random.default_rng(622)
    lens_s, lens_b = rng.integers(1, 65, size=8), rng.integers(1, 129, size=48)
    ids_s, _ = ob.random_token_batch(8, 64, lens_s, seed=623)
    ids_b, _ = ob.random_token_batch(48, 128, lens_b, seed=624)
    ref_small = _bert(w, cfg.to_dict(), "int8").encode(ids_s, lens_s)
    ref_big = _bert(w, cfg.to_dict(), "int8").encode(ids_b, lens_b)
    model = _bert(w, cfg.to_dict(), "int8")
    for _ in range(3):  # direct, capture, replay
        assert np.array_equal(model.encode(ids_s, lens_s), ref_small)
    assert np.array_equal(model.encode(ids_b, lens_b), ref_big)  # workspace grows
    for _ in range(3):
        assert np.array_equal(model.encode(ids_s, lens_s), ref_small)
        assert np.array_equal(model.encode(ids_b, lens_b), ref_big)


# ── post-pool projection head (row (f): fine-tuned embedding adapters) ─────────

@pytest.mark.parametrize("fmt", ["f32", "bf16", "int8"])
def test_projection_head_matches_oracle(fmt, tmp_path):
    """LoraLinear over an identity base on the pooled embedding
    (candle.rs:823-829, 1857-1892): set from arrays, loaded from an adapter
    file, and removed again."""
    from safetensors.numpy import save_file
    cfg, w = _bert_base(631)
    rng = np.random.default_rng(632)
    lens = rng.integers(32, 97, size=12)  # the int8 workload's row lengths (U[32, ...])
    ids, mask = ob.random_token_batch(12, 96, lens, seed=633)
    fwd = oq.bert_int8_forward_hidden if fmt == "int8" else ob.bert_forward_hidden
    pooled = ob.pool_and_normalize(fwd(w, cfg, ids, mask), mask)
    rank, alpha = 8, 16.0
    a = (rng.standard_normal((rank, 768)) * 0.05).astype(np.float32)
    b = (rng.standard_normal((768, rank)) * 0.05).astype(np.float32)
    ref = ob.projection_head(pooled, a, b, alpha)
    model = _bert(w, cfg.to_dict(), fmt)
    plain = model.encode(ids, lens)
    model.set_projection_head(a, b, alpha)
    assert model.info.projection_rank == rank
    assert_close_rows(model.encode(ids, lens), ref, fmt)
    assert_close_rows(model.encode(ids, lens), ref, fmt)  # graph capture keeps the head
    path = tmp_path / "adapter.safetensors"
    save_file({"projection.lora_a": a, "projection.lora_b": b}, str(path))
    model.set_projection_head(None, None, 0.0)
    assert model.info.projection_rank == 0
    assert np.array_equal(model.encode(ids, lens), plain)
    model.load_projection_head(str(path), alpha)
    assert_close_rows(model.encode(ids, lens), ref, fmt)
    empty = tmp_path / "no_head.safetensors"
    save_file({"other": np.zeros(4, np.float32)}, str(empty))
    model.set_projection_head(None, None, 0.0)
    model.load_projection_head(str(empty), alpha)  # the reference's Ok(None)
    assert model.info.projection_rank == 0


# ── LoRA adapters inside the encoder linears (row (f): encoder adapters) ──────

def _lora_set(cfg, seed, ranks, layers, sites=ob.LORA_SITES):
    """{(layer, site): (A [rank, in], B [out, rank], scaling)} at every site of
    `layers`, ranks cycling through `ranks` (odd ones exercise the padding)."""
    rng = np.random.default_rng(seed)
    H, F = cfg.hidden_size, cfg.intermediate_size
    dims = {"query": (H, H), "key": (H, H), "value": (H, H), "dense": (H, H),
            "intermediate_dense": (H, F), "output_dense": (F, H)}
    out, i = {}, 0
    for n in layers:
        for s_name, s_bert in zip(sites, ob.LORA_SITES):
            r = ranks[i % len(ranks)]
            i += 1
            fin, fout = dims[s_bert]
            a = (rng.standard_normal((r, fin)) * (1.0 / np.sqrt(fin))).astype(np.float32)
            b = (rng.standard_normal((fout, r)) * 0.05).astype(np.float32)
            out[(n, s_name)] = (a, b, 16.0 / r)
    return out


@pytest.mark.parametrize("fmt", ["f32", "bf16"])
def test_lora_adapters_match_oracle(fmt, tmp_path):
    """base(x) + scaling (x A^T) B^T at all six linears (LoraLinear,
    lora_linear.rs:226-305; sites of bert.rs:590-640): set from arrays, kept by
    graph replay, removed back to the plain model, loaded from an adapter file
    with alpha / rank and alpha / sqrt(rank) scaling."""
    from safetensors.numpy import save_file
    cfg = ob.BertConfig(256, 4, 4, 1024, 1000, 128)
    w = ob.random_bert_weights(cfg, seed=651)
    rng = np.random.default_rng(652)
    lens = rng.integers(1, 97, size=10)
    lens[0] = 96
    ids, mask = ob.random_token_batch(10, 96, lens, seed=653, id_lo=1, id_hi=999)
    lora = _lora_set(cfg, 654, ranks=[8, 4, 3, 16, 5, 8], layers=[0, 2, 3])
    ref = ob.pool_and_normalize(ob.bert_forward_hidden(w, cfg, ids, mask, lora=lora), mask)
    plain_ref = ob.pool_and_normalize(ob.bert_forward_hidden(w, cfg, ids, mask), mask)
    assert np.abs(ref - plain_ref).max() > 20 * TOL[fmt]  # the adapters matter
    model = _bert(w, cfg.to_dict(), fmt)
    plain = model.encode(ids, lens)
    for (n, site), (a, b, sc) in lora.items():
        model.set_lora(n, site, a, b, sc)
    for _ in range(3):  # direct, capture, replay
        assert_close_rows(model.encode(ids, lens), ref, fmt)
    for (n, site) in lora:
        model.set_lora(n, site, None, None, 0.0)
    assert np.array_equal(model.encode(ids, lens), plain)
    # from an adapter file: scaling alpha / rank, then alpha / sqrt(rank)
    alpha = 12.0
    tensors = {}
    for (n, site), (a, b, _) in lora.items():
        tensors[f"layer.{n}.{site}.lora_a"] = a
        tensors[f"layer.{n}.{site}.lora_b"] = b
    path = tmp_path / "adapter.safetensors"
    save_file(tensors, str(path))
    for rslora in (False, True):
        scaled = {k: (a, b, alpha / (np.sqrt(a.shape[0]) if rslora else a.shape[0]))
                  for k, (a, b, _) in lora.items()}
        ref_f = ob.pool_and_normalize(ob.bert_forward_hidden(w, cfg, ids, mask, lora=scaled), mask)
        assert model.load_lora(str(path), alpha, use_rslora=rslora) == len(lora)
        assert_close_rows(model.encode(ids, lens), ref_f, fmt)


def test_lora_adapters_distilbert():
    """DistilBERT's module names (q_lin .. lin2, distilbert.rs:245-296) from an
    adapter file, against the oracle over the golden fixture's weights."""
    from safetensors.numpy import save_file
    import tempfile
    from jammi_b200 import Bert
    w, g = load_golden("small_distilbert.npz")
    d_cfg = json.loads(bytes(g["config_json"]).decode())
    _, cfg = ob.distilbert_as_bert(w, d_cfg)
    lora = _lora_set(cfg, 661, ranks=[4, 8], layers=range(cfg.num_hidden_layers),
                     sites=ob.DISTILBERT_LORA_SITES)
    ids, mask = g["ids"], g["mask"]
    lens = mask.sum(1)
    ref = ob.pool_and_normalize(ob.distilbert_forward_hidden(w, d_cfg, ids, mask, lora=lora), mask)
    model = Bert.from_weights(w, d_cfg, device=0, fmt="f32", pooling="mean")
    with tempfile.TemporaryDirectory() as d:
        path = f"{d}/adapter.safetensors"
        save_file({f"layer.{n}.{s}.lora_{x}": t for (n, s), (a, b, _) in lora.items()
                   for x, t in (("a", a), ("b", b))}, path)
        # scaling 16 / rank, as _lora_set used
        assert model.load_lora(path, 16.0) == len(lora)
    assert_close_rows(model.encode(ids, lens), ref, "f32")


def test_lora_rejected_in_int8():
    from jammi_b200._lib import JbError
    cfg = ob.BertConfig(64, 1, 2, 128, 100, 32)
    model = _bert(ob.random_bert_weights(cfg, seed=671), cfg.to_dict(), "int8")
    with pytest.raises(JbError):
        model.set_lora(0, "query", np.zeros((4, 64), np.float32), np.zeros((64, 4), np.float32), 1.0)


# ── OpenCLIP text tower (row (f): sibling encoders) ──────────────────────────

def _clip_text(weights, cfg, fmt):
    from jammi_b200 import OpenClipText
    return OpenClipText.from_weights(weights, cfg, device=0, fmt=fmt)


@pytest.mark.parametrize("fmt", ["f32", "bf16"])
def test_clip_text_golden(fmt):
    """ClipText::forward (clip_text.rs:296-331) against HF
    CLIPTextModelWithProjection: causal blocks, EOT pooling, text_projection, L2."""
    w, g = load_golden("small_clip_text.npz")
    cfg = json.loads(bytes(g["config_json"]).decode())
    model = _clip_text(w, cfg, fmt)
    assert model.embed_dim() == 32 and model.context_length() == 24
    for _ in range(3):  # direct, capture, replay
        assert_close_rows(model.encode(g["ids"]), g["embed"], fmt)


def test_clip_text_vit_b32_bf16_config():
    """The ViT-B/32 text tower (width 512, 12 layers, 8 heads, context 77,
    vocab 49408, embed 512), bf16, ragged EOT positions."""
    cfg = oc.ClipTextConfig()
    w = oc.random_clip_text_weights(cfg, seed=701, std=0.05)
    rng = np.random.default_rng(702)
    lens = rng.integers(2, 78, size=24)
    lens[:3] = [77, 2, 3]
    ids = oc.random_clip_text_batch(24, 77, lens, seed=703, vocab=cfg.vocab_size)
    ref = oc.clip_text_forward(w, cfg, ids)
    model = _clip_text(w, cfg.to_open_clip_config(), "bf16")
    assert_close_rows(model.encode(ids), ref, "bf16")
    # ids after the EOT token are never computed: the output does not move
    noisy = ids.copy()
    for b, n in enumerate(lens):
        noisy[b, n:] = rng.integers(1, cfg.vocab_size - 2, size=77 - n)
    assert np.array_equal(model.encode(noisy), model.encode(ids))
    # a shorter padded width gives the same rows (positions are absolute)
    short = ids[3:, :int(lens[3:].max())]
    np.testing.assert_allclose(model.encode(short), model.encode(ids)[3:], rtol=0, atol=2e-6)


def test_clip_text_errors():
    from jammi_b200 import SequenceTooLong
    from jammi_b200._lib import JbError
    w, g = load_golden("small_clip_text.npz")
    cfg = json.loads(bytes(g["config_json"]).decode())
    model = _clip_text(w, cfg, "f32")
    with pytest.raises(SequenceTooLong):  # clip_text.rs:302-308
        model.encode(np.zeros((1, 25), np.uint32))
    bad = g["ids"].copy()
    bad[0, 0] = 300  # vocab 300
    with pytest.raises(JbError):
        model.encode(bad)
    with pytest.raises(JbError):  # text towers carry no projection head or LoRA sites here
        model.set_lora(0, "query", np.zeros((4, 64), np.float32), np.zeros((64, 4), np.float32), 1.0)


# ── ModernBERT (row (f): sibling encoders) ────────────────────────────────────

@pytest.mark.parametrize("fmt", ["f32", "bf16"])
def test_modernbert_golden(fmt):
    """ModernBert (modernbert.rs): RoPE on Q/K, GeGLU, bias-free pre-norm layers,
    against HF ModernBertModel, all poolings and the hidden states."""
    from jammi_b200 import Bert
    from jammi_b200._lib import TEXT_MODERNBERT
    w, g = load_golden("small_modernbert.npz")
    cfg = json.loads(bytes(g["config_json"]).decode())
    model = Bert.from_weights(w, cfg, device=0, fmt=fmt)
    assert model.info.variant == TEXT_MODERNBERT
    lens = g["mask"].sum(1)
    for pname in ("mean", "cls", "max", "weighted_mean"):
        out = model.encode(g["ids"], lens, pooling=pname)
        rows = lens > 0 if pname == "cls" else None
        assert_close_rows(out, g["pooled_" + pname], fmt, rows)
    assert np.all(model.encode(g["ids"], lens)[lens == 0] == 0)
    h = model.forward_hidden(g["ids"], g["mask"]).cpu().numpy()
    valid = g["mask"].astype(bool)
    bar = 1e-4 if fmt == "f32" else 6e-2  # hidden states of magnitude ~1-4
    assert np.abs(h[valid] - g["hidden"][valid]).max() <= bar
    assert np.all(h[~valid] == 0)


def test_modernbert_base_bf16_config():
    """ModernBERT-base dimensions (H 768, 22 layers, 12 heads, GeGLU 1152,
    vocab 50368), bf16, ragged rows, against the oracle."""
    cfg = {"model_type": "modernbert", "hidden_size": 768, "num_hidden_layers": 22,
           "num_attention_heads": 12, "intermediate_size": 1152, "vocab_size": 50368,
           "max_position_embeddings": 8192, "global_rope_theta": 160000.0}
    w = ob.random_modernbert_weights(cfg, seed=811)
    rng = np.random.default_rng(812)
    lens = rng.integers(1, 201, size=10)
    lens[0] = 200
    ids, mask = ob.random_token_batch(10, 200, lens, seed=813, id_lo=1, id_hi=50367, cls_id=1, sep_id=2)
    ref = ob.pool_and_normalize(ob.modernbert_forward_hidden(w, cfg, ids, mask), mask)
    from jammi_b200 import Bert
    model = Bert.from_weights(w, cfg, device=0, fmt="bf16")
    assert_close_rows(model.encode(ids, lens), ref, "bf16")


def test_modernbert_refusals():
    from jammi_b200 import Bert
    from jammi_b200._lib import JbError
    w, g = load_golden("small_modernbert.npz")
    cfg = json.loads(bytes(g["config_json"]).decode())
    with pytest.raises(JbError):  # no int8 ModernBERT weights
        Bert.from_weights(w, cfg, device=0, fmt="int8")
    model = Bert.from_weights(w, cfg, device=0, fmt="bf16")
    with pytest.raises(JbError):
        model.set_lora(0, "query", np.zeros((4, 64), np.float32), np.zeros((64, 4), np.float32), 1.0)


# ── device image preprocessing in the image entry point (row (f): host preprocessing) ──

def test_encode_rgb8_matches_preprocessed_pixels():
    """jb_encode_image_rgb8 (raw RGB8 bytes in, preprocessing on the device)
    equals jb_encode_image on the oracle's preprocessed pixels, bit for bit."""
    from oracle import image as oimg
    from jammi_b200 import OpenClipVisionTransformer
    w, g = load_golden("tiny_clip_cls.npz")
    cfg = json.loads(bytes(g["config_json"]).decode())
    cfg["preprocess_cfg"] = {"mean": [0.5, 0.4, 0.3], "std": [0.2, 0.25, 0.3]}
    model = OpenClipVisionTransformer.from_weights(w, cfg, device=0, fmt="f32")
    assert np.allclose(list(model.info.preprocess_mean), [0.5, 0.4, 0.3])
    imgs = oimg.random_images(21, [(40, 20), (8, 8), (3, 11), (100, 100), (9, 64)])
    px = oimg.preprocess_image_batch(imgs, model.image_size(), (0.5, 0.4, 0.3), (0.2, 0.25, 0.3))
    for _ in range(3):  # direct, capture, replay
        assert np.array_equal(model.encode_rgb8(imgs), model.forward_image(px))
    with pytest.raises(Exception):
        model.encode_rgb8([np.zeros((0, 4, 3), np.uint8)])


def test_embed_images_null_rows_match_direct_calls():
    """driver.embed_images: null images are zero rows with validity 0, the
    others equal jb_encode_image_rgb8 on the same images, bit for bit."""
    from oracle import image as oimg
    from jammi_b200 import OpenClipVisionTransformer
    from jammi_b200.driver import embed_images
    w, g = load_golden("tiny_clip_cls.npz")
    cfg = json.loads(bytes(g["config_json"]).decode())
    model = OpenClipVisionTransformer.from_weights(w, cfg, device=0, fmt="f32")
    imgs = oimg.random_images(5, [(40, 20), (8, 8), (3, 11), (100, 100), (9, 64)])
    rows = [imgs[0], None, imgs[1], imgs[2], None, imgs[3], imgs[4]]
    out, valid = embed_images(model, rows, batch_rows=2)
    want = model.encode_rgb8(imgs)
    assert np.array_equal(out[[0, 2, 3, 5, 6]], want)
    assert not out[[1, 4]].any()
    assert np.unpackbits(valid, bitorder="little")[:7].tolist() == [1, 0, 1, 1, 0, 1, 1]
