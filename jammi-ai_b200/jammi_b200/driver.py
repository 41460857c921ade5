"""Host runtime bindings: memory-budget admission, the chunked runner and the
multi-device embedding driver (all implemented in C++ inside the library).

* ``Scheduler``            -- ``GpuScheduler`` (crates/jammi-ai/src/concurrency/gpu_scheduler.rs)
* ``run_chunks``           -- ``InferenceRunner::run_chunks`` with OOM halving
  (crates/jammi-ai/src/inference/runner.rs:176-256)
* ``generate_embeddings``  -- the ``generate_embeddings`` driver over one model
  handle per device, row-order output in Arrow FixedSizeList layout.
* ``embed_texts``          -- the same over text, tokenisation off the critical
  path: a producer thread tokenises chunk k + 1 while the devices embed chunk k
  (the embedding pipeline's tokenise -> forward loop, crates/jammi-ai/src/
  pipeline/embedding.rs:47-282 with tokenizer.rs:45-93, overlapped).
"""
from __future__ import annotations

import ctypes
import queue
import threading

import numpy as np

from . import _lib as L
from ._lib import JbError, check, lib
from .encoders import POOLING


class GenerateOpts(ctypes.Structure):
    _fields_ = [("batch_rows", ctypes.c_int32), ("pooling", ctypes.c_int32),
                ("sort_by_length", ctypes.c_int32), ("pad_multiple", ctypes.c_int32),
                ("memory_fraction", ctypes.c_double)]


class GenerateStats(ctypes.Structure):
    _fields_ = [("rows", ctypes.c_int64), ("valid_rows", ctypes.c_int64), ("batches", ctypes.c_int64),
                ("tokens", ctypes.c_int64), ("oom_retries", ctypes.c_int64), ("seconds", ctypes.c_double),
                ("h2d_bytes", ctypes.c_int64), ("d2h_bytes", ctypes.c_int64),
                ("prepare_seconds", ctypes.c_double), ("pack_seconds", ctypes.c_double),
                ("scatter_seconds", ctypes.c_double), ("wait_seconds", ctypes.c_double),
                ("worker_seconds_max", ctypes.c_double), ("worker_seconds_min", ctypes.c_double),
                ("enqueue_seconds", ctypes.c_double), ("setup_seconds", ctypes.c_double)]


FORWARD_CB = ctypes.CFUNCTYPE(ctypes.c_int, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64,
                              ctypes.c_void_p, ctypes.c_size_t)


class Scheduler:
    """GPU memory-budget admission (one per device)."""

    def __init__(self, handle):
        if not handle:
            msg = lib().jb_last_error()
            raise JbError(L.ERR_INVALID, msg.decode() if msg else "scheduler creation failed")
        self._h = ctypes.c_void_p(handle)

    @classmethod
    def new(cls, total_bytes: int, headroom_fraction: float):
        return cls(lib().jb_scheduler_new(int(total_bytes), float(headroom_fraction)))

    @classmethod
    def unlimited(cls):
        return cls(lib().jb_scheduler_new_unlimited())

    @classmethod
    def for_device(cls, device: int, memory_fraction: float):
        return cls(lib().jb_scheduler_for_device(int(device), float(memory_fraction)))

    @property
    def is_unlimited(self) -> bool:
        return bool(lib().jb_scheduler_is_unlimited(self._h))

    def available(self) -> int:
        return int(lib().jb_scheduler_available(self._h))

    def try_acquire(self, nbytes: int) -> bool:
        return bool(lib().jb_scheduler_try_acquire(self._h, int(nbytes)))

    def acquire(self, nbytes: int, priority: int = 0, timeout_ms: int = -1):
        check(lib().jb_scheduler_acquire(self._h, int(nbytes), int(priority), int(timeout_ms)))

    def release(self, nbytes: int):
        lib().jb_scheduler_release(self._h, int(nbytes))

    def close(self):
        if getattr(self, "_h", None):
            lib().jb_scheduler_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def is_oom_message(msg: str) -> bool:
    return bool(lib().jb_is_oom_message(msg.encode()))


def run_chunks(rows: int, batch_size: int, forward) -> int:
    """Run ``forward(start, count)`` over ``rows`` in chunks; an exception whose
    text is an OOM halves the batch and retries the same slice.  Returns the
    final batch size; raises JbError for a propagated failure."""
    def cb(_user, start, count, msg, msg_len):
        try:
            forward(int(start), int(count))
            return L.OK
        except Exception as e:  # noqa: BLE001 -- the message crosses the ABI
            text = str(e).encode()[: max(0, int(msg_len) - 1)]
            ctypes.memmove(msg, text + b"\0", len(text) + 1)
            return int(getattr(e, "status", L.ERR_INVALID))
    c_cb = FORWARD_CB(cb)
    bs = ctypes.c_int(int(batch_size))
    check(lib().jb_run_chunks(int(rows), ctypes.byref(bs), ctypes.cast(c_cb, ctypes.c_void_p), None))
    return bs.value


def pack_rows(rows) -> tuple[np.ndarray, np.ndarray]:
    """List of token-id sequences -> (values u32, offsets u64[len+1])."""
    lens = np.array([len(r) for r in rows], dtype=np.uint64)
    offsets = np.zeros(len(rows) + 1, dtype=np.uint64)
    np.cumsum(lens, out=offsets[1:])
    values = np.concatenate([np.asarray(r, dtype=np.uint32) for r in rows]) if len(rows) else np.zeros(0, np.uint32)
    return np.ascontiguousarray(values, dtype=np.uint32), offsets


def generate_embeddings(models, values, offsets, batch_rows: int = 256, pooling: str = "mean",
                        sort_by_length: bool = True, pad_multiple: int = 8,
                        memory_fraction: float = 0.0, out=None, validity=None):
    """Embeddings for every row, in row order.  ``models``: one Bert per device.
    Returns (out f32 [rows, H], validity bitmap u8 [(rows+7)//8], stats dict).
    ``out`` / ``validity`` may be caller-owned buffers of those shapes (reused
    across calls, their pages already mapped)."""
    values = np.ascontiguousarray(values, dtype=np.uint32)
    offsets = np.ascontiguousarray(offsets, dtype=np.uint64)
    rows = offsets.size - 1
    H = models[0].info.output_dim
    if out is None:
        out = np.empty((rows, H), dtype=np.float32)
    elif out.dtype != np.float32 or out.shape != (rows, H) or not out.flags.c_contiguous:
        raise ValueError("out must be a C-contiguous float32 [rows, hidden] array")
    if validity is None:
        validity = np.zeros((rows + 7) // 8, dtype=np.uint8)
    elif validity.dtype != np.uint8 or validity.size != (rows + 7) // 8 or not validity.flags.c_contiguous:
        raise ValueError("validity must be a C-contiguous uint8 [(rows + 7) // 8] array")
    handles = (ctypes.c_void_p * len(models))(*[m.handle.value for m in models])
    opts = GenerateOpts(int(batch_rows), POOLING[pooling], 1 if sort_by_length else 0,
                        int(pad_multiple), float(memory_fraction))
    stats = GenerateStats()
    vp = values.ctypes.data if values.size else None
    check(lib().jb_generate_embeddings(handles, len(models), vp, offsets.ctypes.data, rows,
                                       ctypes.byref(opts), out.ctypes.data, validity.ctypes.data,
                                       ctypes.byref(stats)))
    st = {k: getattr(stats, k) for k, _ in GenerateStats._fields_}
    return out, validity, st


def generate_embeddings_stream(models, row_chunks, **kw):
    """``generate_embeddings`` over an iterable of row chunks (lists of token-id
    sequences), producing chunk k + 1 on a background thread while chunk k is
    embedded (the C driver releases the GIL).  Yields (out, validity, stats)
    per chunk, in order."""
    q: queue.Queue = queue.Queue(maxsize=2)
    done = object()
    failure = []

    def produce():
        try:
            for rows in row_chunks:
                q.put(pack_rows(rows))
        except BaseException as e:  # handed to the consumer
            failure.append(e)
        finally:
            q.put(done)

    t = threading.Thread(target=produce, name="jb-tokenize", daemon=True)
    t.start()
    try:
        while True:
            item = q.get()
            if item is done:
                break
            values, offsets = item
            yield generate_embeddings(models, values, offsets, **kw)
    finally:
        # let a blocked producer finish, then join it
        while t.is_alive():
            try:
                q.get_nowait()
            except queue.Empty:
                t.join(timeout=0.01)
    if failure:
        raise failure[0]


def embed_texts(models, texts, tokenize, chunk_rows: int = 65536, **kw):
    """Embeddings of ``texts`` in order: ``tokenize(list_of_texts)`` returns one
    token-id sequence per text (e.g. a wrapped HF tokenizer's ``input_ids``,
    [CLS] ... [SEP]); it runs on a producer thread one chunk ahead of the
    devices.  As ``CandleModel::forward_embedding`` (candle.rs:764-856): an
    empty or None text is a null row (zero vector, validity 0) and never
    reaches the tokenizer, and a library ``Tokenizer`` without its own
    max_length truncates to the model's max sequence length (a caller's own
    callable must truncate itself).  Returns (out f32 [rows, H], validity
    bitmap, list of per-chunk stats)."""
    if chunk_rows <= 0:
        raise ValueError("chunk_rows must be positive")
    texts = list(texts)
    H = models[0].info.output_dim
    from .tokenizer import Tokenizer
    if isinstance(tokenize, Tokenizer):
        max_len = tokenize.max_length if tokenize.max_length > 0 else int(models[0].info.max_seq)
        base = tokenize

        def tokenize_valid(chunk):  # jb_tokenize_rows: null rows in C, on all host cores
            ids, offs = base.encode_ragged(chunk, max_length=max_len, null_rows=True)
            return [ids[offs[i]:offs[i + 1]] for i in range(len(chunk))]
    else:
        def tokenize_valid(chunk):
            keep = [i for i, t in enumerate(chunk)
                    if t is not None and not (isinstance(t, (str, bytes)) and len(t) == 0)]
            seqs = tokenize([chunk[i] for i in keep]) if keep else []
            rows = [[] for _ in chunk]
            for i, seq in zip(keep, seqs):
                rows[i] = seq
            return rows

    chunks = (tokenize_valid(texts[i:i + chunk_rows]) for i in range(0, len(texts), chunk_rows))
    outs, valid, stats = [], [], []
    for out, validity, st in generate_embeddings_stream(models, chunks, **kw):
        outs.append(out)
        valid.append(np.unpackbits(validity, bitorder="little")[: out.shape[0]])
        stats.append(st)
    if not outs:
        return np.zeros((0, H), np.float32), np.zeros(0, np.uint8), stats
    bits = np.concatenate(valid)
    if bits.size and not bits.any():
        # the all-invalid guard of EmbeddingPipeline::run (embedding.rs:204-230):
        # a job whose every row is empty produces no table, loudly
        raise JbError(L.ERR_INVALID, "embedding generation produced no embeddings: every input row "
                                     "was empty or invalid (no valid content to embed)")
    return np.concatenate(outs), np.packbits(bits, bitorder="little"), stats


def embed_images(model, images, batch_rows: int = 512):
    """``CandleModel::forward_image_embedding`` (candle.rs:858-937) over decoded
    RGB8 images (``[h, w, 3]`` uint8 arrays, preprocessing on the device): a
    None entry (a null image) is a null row -- zero vector, validity 0 -- and
    never reaches the device; a job of only null images is an error.  Returns
    (out f32 [rows, embed_dim], validity bitmap)."""
    if batch_rows <= 0:
        raise ValueError("batch_rows must be positive")
    images = list(images)
    out = np.zeros((len(images), model.info.output_dim), np.float32)
    valid = np.zeros(len(images), np.uint8)
    keep = [i for i, im in enumerate(images) if im is not None]
    if images and not keep:  # EmbeddingPipeline::run's all-invalid guard (embedding.rs:204-230)
        raise JbError(L.ERR_INVALID, "embedding generation produced no embeddings: every input row "
                                     "was empty or invalid (no valid content to embed)")
    for s in range(0, len(keep), batch_rows):
        idx = keep[s:s + batch_rows]
        out[idx] = model.encode_rgb8([images[i] for i in idx])
        valid[idx] = 1
    return out, np.packbits(valid, bitorder="little")
