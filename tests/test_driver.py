"""Host runtime on CPU: the memory-budget scheduler and the chunked runner,
restating the reference's own tests with fakes (no GPU needed):
crates/jammi-ai/tests/it/scheduling.rs, crates/jammi-ai/src/concurrency/gpu_scheduler.rs:221-266,
crates/jammi-ai/src/inference/runner.rs:297-502."""
import threading
import time

import pytest

from jammi_b200 import _lib as L
from jammi_b200.driver import Scheduler, is_oom_message, run_chunks
from jammi_b200._lib import JbError

GB = 1_000_000_000


# ── scheduler ───────────────────────────────────────────────────────────────

def test_permit_lifecycle_and_release():
    s = Scheduler.new(GB, 0.2)
    initial = s.available()
    assert initial == 800_000_000
    assert s.try_acquire(300_000_000)
    assert s.available() == initial - 300_000_000
    s.release(300_000_000)
    assert s.available() == initial


def test_headroom_fraction_enforced():
    s = Scheduler.new(GB, 0.2)
    assert s.try_acquire(800_000_000), "exact usable limit must succeed"
    assert s.available() == 0
    assert not s.try_acquire(1)
    s.release(800_000_000)
    assert s.available() == 800_000_000
    half = Scheduler.new(GB, 0.5)
    assert half.available() == 500_000_000
    assert not half.try_acquire(600_000_000)
    assert half.try_acquire(500_000_000)


def test_headroom_out_of_range_rejected():
    with pytest.raises(JbError):
        Scheduler.new(GB, 1.5)


def test_unlimited_and_cpu_device():
    u = Scheduler.unlimited()
    assert u.is_unlimited and u.available() == 2**64 - 1
    assert u.try_acquire(10**18)
    assert Scheduler.for_device(-1, 0.9).is_unlimited


def test_for_device_probe_failure_is_unlimited():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present: the probe succeeds")
    assert Scheduler.for_device(0, 0.9).is_unlimited


def test_blocking_acquire_wakes_on_release():
    s = Scheduler.new(GB, 0.0)
    assert s.try_acquire(900_000_000)
    got = threading.Event()

    def waiter():
        s.acquire(500_000_000, timeout_ms=10_000)
        got.set()

    t = threading.Thread(target=waiter)
    t.start()
    time.sleep(0.05)
    assert not got.is_set(), "must block while the budget is exhausted"
    s.release(900_000_000)
    t.join(5)
    assert got.is_set()
    assert s.available() == 500_000_000


def test_acquire_timeout_and_oversize():
    s = Scheduler.new(GB, 0.0)
    assert s.try_acquire(GB)
    with pytest.raises(JbError) as e:
        s.acquire(1, timeout_ms=50)
    assert e.value.status == L.ERR_TIMEOUT
    with pytest.raises(JbError) as e:
        s.acquire(2 * GB, timeout_ms=50)
    assert e.value.status == L.ERR_OOM and "out of memory" in str(e.value)


def test_concurrent_acquire_stress_and_liveness():
    s = Scheduler.new(GB, 0.1)
    usable = s.available()
    permit = 100_000_000
    violations = []

    def task():
        for _ in range(50):
            s.acquire(permit, timeout_ms=10_000)
            if s.available() > usable - permit:
                violations.append(s.available())
            s.release(permit)

    ts = [threading.Thread(target=task) for _ in range(16)]
    for t in ts:
        t.start()
    for t in ts:
        t.join(30)
    assert not violations
    assert s.available() == usable


# ── runner ──────────────────────────────────────────────────────────────────

class FakeOom(Exception):
    status = L.ERR_OOM


def test_oom_classifier():
    for msg in ("CUDA out of memory", "CUDA_ERROR_OUT_OF_MEMORY", "OutOfMemory", "oom killer"):
        assert is_oom_message(msg)
    for msg in ("CUDA_ERROR_INVALID_PTX", "cuda launch failed", "shape mismatch"):
        assert not is_oom_message(msg)


def test_row_conservation_across_oom_halving():
    seen = []

    def forward(start, count):
        if count > 37:
            raise FakeOom("CUDA out of memory: tried to allocate")
        seen.extend(range(start, start + count))

    bs = run_chunks(300, 256, forward)
    assert seen == list(range(300)), "no row skipped or duplicated"
    assert bs == 32


def test_persistent_oom_at_batch_one_propagates():
    calls = []

    def forward(start, count):
        calls.append(count)
        raise FakeOom("out of memory")

    with pytest.raises(JbError) as e:
        run_chunks(10, 8, forward)
    assert calls == [8, 4, 2, 1]
    assert "out of memory" in str(e.value)


def test_non_oom_error_propagates_immediately():
    calls = []

    class Broken(Exception):
        status = L.ERR_CUDA

    def forward(start, count):
        calls.append(count)
        raise Broken("CUDA_ERROR_INVALID_PTX")

    with pytest.raises(JbError) as e:
        run_chunks(100, 16, forward)
    assert calls == [16], "a systemic error is never retried"
    assert e.value.status == L.ERR_CUDA


# ── tokenisation overlapped with the devices (embed_texts) ───────────────────

def test_stream_tokenises_ahead_in_order(monkeypatch):
    """The producer thread runs one chunk ahead of the embedding calls; chunks
    come back in order, and a tokenizer failure reaches the caller."""
    import numpy as np
    from jammi_b200 import driver as D
    calls, produced = [], []

    def fake_generate(models, values, offsets, **kw):
        rows = offsets.size - 1
        calls.append((len(produced), rows))
        time.sleep(0.02)
        out = np.tile(np.arange(rows, dtype=np.float32)[:, None], (1, 4)) + values[:1].sum()
        return out, np.full((rows + 7) // 8, 0xFF, np.uint8), {"rows": rows}

    def tokenize(texts):
        produced.append(len(texts))
        return [[int(t)] * (1 + int(t) % 3) for t in texts]

    monkeypatch.setattr(D, "generate_embeddings", fake_generate)

    class M:
        class info:
            hidden = 4
            output_dim = 4
    out, valid, stats = D.embed_texts([M()], [str(i) for i in range(10)], tokenize, chunk_rows=4)
    assert [st["rows"] for st in stats] == [4, 4, 2]
    assert out.shape == (10, 4)
    assert np.array_equal(np.unpackbits(valid, bitorder="little")[:10], np.ones(10, np.uint8))
    # by the time chunk k is embedded, chunk k + 1 has usually been tokenised
    assert calls[0][0] >= 1

    def bad(texts):
        raise RuntimeError("tokenizer failed")
    with pytest.raises(RuntimeError):
        D.embed_texts([M()], ["a", "b"], bad, chunk_rows=1)


def test_embed_texts_with_the_library_tokenizer(monkeypatch, tmp_path):
    """The library's Tokenizer is a tokenize callable for embed_texts."""
    import numpy as np
    pytest.importorskip("tokenizers")
    from test_tokenizer import build
    from jammi_b200 import Tokenizer
    from jammi_b200 import driver as D
    hf, path = build(tmp_path, "tok.json")
    seen = []

    def fake_generate(models, values, offsets, **kw):
        seen.append((values.copy(), offsets.copy()))
        rows = offsets.size - 1
        bits = np.packbits((np.diff(offsets.astype(np.int64)) > 0).astype(np.uint8), bitorder="little")
        return np.zeros((rows, 4), np.float32), bits, {"rows": rows}

    monkeypatch.setattr(D, "generate_embeddings", fake_generate)

    class M:
        class info:
            hidden = 4
            output_dim = 4
            max_seq = 6
    texts = ["hello world", "naïve café", "", "東京", None, "a b c d e f g h"]
    _, valid, _ = D.embed_texts([M()], texts, Tokenizer(path), chunk_rows=3)
    ids = np.concatenate([v for v, _ in seen])
    # empty / None texts are null rows that never reach the tokenizer; the
    # rest are truncated to the model's max_seq (candle.rs:779-806)
    hf.enable_truncation(max_length=6)
    want = np.concatenate([np.array(e.ids, np.uint32) for e in hf.encode_batch([t for t in texts if t])])
    assert np.array_equal(ids, want)
    assert np.unpackbits(valid, bitorder="little")[:6].tolist() == [1, 1, 0, 1, 0, 1]


def test_embed_texts_all_invalid_rows_fail_loudly(monkeypatch):
    """EmbeddingPipeline::run's all-invalid guard (embedding.rs:204-230): every
    row empty -> an error, not a silently empty result; one valid row is
    enough to succeed (the empty ones stay null)."""
    import numpy as np
    from jammi_b200 import driver as D
    from jammi_b200._lib import JbError

    def fake_generate(models, values, offsets, **kw):
        rows = offsets.size - 1
        lens = np.diff(offsets.astype(np.int64))
        bits = np.packbits((lens > 0).astype(np.uint8), bitorder="little")
        return np.zeros((rows, 4), np.float32), bits, {"rows": rows}

    monkeypatch.setattr(D, "generate_embeddings", fake_generate)

    class M:
        class info:
            hidden = 4
            output_dim = 4
    with pytest.raises(JbError, match="no embeddings"):
        D.embed_texts([M()], ["", "", ""], lambda ts: [[] for _ in ts], chunk_rows=2)
    out, valid, _ = D.embed_texts([M()], ["", "x", ""], lambda ts: [[7] if t else [] for t in ts], chunk_rows=2)
    assert np.unpackbits(valid, bitorder="little")[:3].tolist() == [0, 1, 0]
    assert D.embed_texts([M()], [], lambda ts: [], chunk_rows=2)[0].shape == (0, 4)


def test_embed_images_null_rows():
    """forward_image_embedding's row rules (candle.rs:880-893): a null image is
    a null row that never reaches the device; the rest keep their order."""
    import numpy as np
    from jammi_b200 import driver as D
    seen = []

    class M:
        class info:
            output_dim = 3

        def encode_rgb8(self, imgs):
            seen.append(len(imgs))
            return np.array([[im.shape[0], im.shape[1], 1.0] for im in imgs], np.float32)
    imgs = [np.zeros((2, 5, 3), np.uint8), None, np.zeros((7, 1, 3), np.uint8), None,
            np.zeros((4, 4, 3), np.uint8)]
    out, valid = D.embed_images(M(), imgs, batch_rows=2)
    assert seen == [2, 1]
    assert out.tolist() == [[2, 5, 1], [0, 0, 0], [7, 1, 1], [0, 0, 0], [4, 4, 1]]
    assert np.unpackbits(valid, bitorder="little")[:5].tolist() == [1, 0, 1, 0, 1]
    from jammi_b200._lib import JbError
    with pytest.raises(JbError, match="no embeddings"):
        D.embed_images(M(), [None, None])
    assert seen == [2, 1]
    assert D.embed_images(M(), [])[0].shape == (0, 3)
