"""Python mirror of the reference's encoder surface over the C ABI.

* ``Bert``                       -- ``jammi_encoders::Bert``
  (crates/jammi-encoders/src/bert.rs): ``forward`` (pooled, L2-normalised),
  ``forward_hidden``, ``hidden_size``, ``max_seq_length``, ``SequenceTooLong``.
* ``OpenClipVisionTransformer``  -- crates/jammi-ai/src/model/backend/open_clip_vit.rs
  with the caller's ``l2_normalize`` (candle.rs:425-438).
* ``OpenClipText``               -- crates/jammi-encoders/src/clip_text.rs (the
  OpenCLIP text tower, ``OpenClipTextForward`` in open_clip_text.rs).
* ``load_model``                 -- ``CandleBackend::load`` for these families.

All compute runs in libjammi_b200.so on the GPU; numpy/torch only carry
buffers across the boundary.
"""
from __future__ import annotations

import ctypes
import json
import os
import tempfile

import numpy as np

from . import _lib as L
from ._lib import JbError, check, lib

POOLING = {"mean": L.POOL_MEAN, "cls": L.POOL_CLS, "max": L.POOL_MAX,
           "weighted_mean": L.POOL_WEIGHTED_MEAN}


class SequenceTooLong(JbError):
    """``EncoderError::SequenceTooLong`` (bert.rs:263-268)."""


def _ptr(a) -> int:
    if hasattr(a, "data_ptr"):
        return a.data_ptr()
    return a.ctypes.data


def _stream_ptr(stream) -> int:
    if stream is None:
        return 0
    return int(getattr(stream, "cuda_stream", stream))


class Model:
    """An owned jb_model handle bound to one device."""

    FAMILY = -1  # detected from the config

    def __init__(self, weights_path: str, config: dict | str, device: int = 0,
                 fmt: str = "bf16"):
        cfg = config if isinstance(config, str) else json.dumps(config)
        h = ctypes.c_void_p()
        check(lib().jb_model_load_family(weights_path.encode(), cfg.encode(), int(device),
                                         L.FORMATS[fmt], self.FAMILY, ctypes.byref(h)))
        self._h = h
        self.info = self._info()
        self.device = device
        self.fmt = fmt

    def _info(self):
        info = L.ModelInfo()
        check(lib().jb_model_get_info(self._h, ctypes.byref(info)))
        return info

    @classmethod
    def from_weights(cls, weights: dict, config: dict, device: int = 0, fmt: str = "bf16"):
        """Write ``weights`` (name -> numpy array) to a temporary safetensors
        file and load it (the file is removed once the weights are on device)."""
        from safetensors.numpy import save_file
        fd, path = tempfile.mkstemp(suffix=".safetensors")
        os.close(fd)
        try:
            save_file({k: np.ascontiguousarray(v) for k, v in weights.items()}, path)
            return cls(path, config, device, fmt)
        finally:
            os.unlink(path)

    def close(self):
        if getattr(self, "_h", None):
            lib().jb_model_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def handle(self):
        return self._h

    def estimate_batch_bytes(self, batch: int, seq: int) -> int:
        return int(lib().jb_estimate_batch_bytes(self._h, batch, seq))

    def sync(self, stream=None):
        check(lib().jb_model_sync(self._h, _stream_ptr(stream)))

    def set_projection_head(self, lora_a, lora_b, lora_alpha: float):
        """Install the post-pool projection head y = x + (alpha/rank) (x A^T) B^T
        (``jb_model_set_projection_head``); ``lora_a`` [rank, H], ``lora_b`` [H, rank].
        ``lora_a=None`` removes it."""
        if lora_a is None:
            check(lib().jb_model_set_projection_head(self._h, None, None, 0, float(lora_alpha)))
        else:
            a = np.ascontiguousarray(lora_a, dtype=np.float32)
            b = np.ascontiguousarray(lora_b, dtype=np.float32)
            check(lib().jb_model_set_projection_head(self._h, a.ctypes.data, b.ctypes.data,
                                                     int(a.shape[0]), float(lora_alpha)))
        self.info = self._info()

    def load_projection_head(self, adapter_path: str, lora_alpha: float):
        """``jb_model_load_projection_head``: from an adapter safetensors file."""
        check(lib().jb_model_load_projection_head(self._h, str(adapter_path).encode(), float(lora_alpha)))
        self.info = self._info()

    LORA_SITES = ("query", "key", "value", "dense", "intermediate_dense", "output_dense")

    def set_lora(self, layer: int, site, lora_a, lora_b, scaling: float):
        """``jb_model_set_lora``: base(x) + scaling (x A^T) B^T at one linear.
        ``site`` is an index or a name of ``LORA_SITES``; ``lora_a=None``
        removes the adapter."""
        s = self.LORA_SITES.index(site) if isinstance(site, str) else int(site)
        if lora_a is None:
            check(lib().jb_model_set_lora(self._h, int(layer), s, None, None, 0, float(scaling)))
            return
        a = np.ascontiguousarray(lora_a, dtype=np.float32)
        b = np.ascontiguousarray(lora_b, dtype=np.float32)
        check(lib().jb_model_set_lora(self._h, int(layer), s, a.ctypes.data, b.ctypes.data,
                                      int(a.shape[0]), float(scaling)))

    def load_lora(self, adapter_path: str, lora_alpha: float, use_rslora: bool = False) -> int:
        """``jb_model_load_lora``: every ``layer.{n}.{module}.lora_a/b`` of an
        adapter file; returns the number of sites installed."""
        n = ctypes.c_int32(0)
        check(lib().jb_model_load_lora(self._h, str(adapter_path).encode(), float(lora_alpha),
                                       1 if use_rslora else 0, ctypes.byref(n)))
        return n.value

    def profile_enable(self, on: bool = True):
        check(lib().jb_model_profile_enable(self._h, 1 if on else 0))

    def profile_read(self) -> dict:
        """Summed device ms and launch counts per kernel class since enable."""
        ms = (ctypes.c_double * 3)()
        n = (ctypes.c_int32 * 3)()
        check(lib().jb_model_profile_read(self._h, ms, n))
        names = ("linear", "attention", "memory")
        return {k: {"ms": ms[i], "launches": n[i]} for i, k in enumerate(names)}


def _raise_seq(e: JbError):
    if e.status == L.ERR_SEQ_TOO_LONG:
        raise SequenceTooLong(e.status, str(e)) from None
    raise e


def mask_to_lengths(mask) -> np.ndarray:
    """The attention mask of ``BatchEncoding`` is a prefix of ones per row
    (right padding, crates/jammi-ai/src/model/tokenizer.rs:82-93); lengths
    are its row sums.  Masks with holes are rejected."""
    m = np.asarray(mask).astype(np.uint32)
    lens = m.sum(axis=1).astype(np.uint32)
    S = m.shape[1]
    prefix = (np.arange(S)[None, :] < lens[:, None]).astype(np.uint32)
    if not np.array_equal(prefix, m):
        raise ValueError("attention mask must be a prefix of ones per row (right padding)")
    return lens


class Bert(Model):
    """``jammi_encoders::Bert`` on the B200 library."""

    def __init__(self, *a, pooling: str = "mean", **kw):
        super().__init__(*a, **kw)
        if self.info.family != L.FAMILY_BERT:
            raise JbError(L.ERR_INVALID, "not a BERT checkpoint")
        self.pooling = pooling

    @classmethod
    def from_weights(cls, weights, config, device=0, fmt="bf16", pooling="mean"):
        m = super().from_weights(weights, config, device, fmt)
        m.pooling = pooling
        return m

    def hidden_size(self) -> int:
        return self.info.hidden

    def max_seq_length(self) -> int:
        return self.info.max_seq

    def encode(self, ids, lens, pooling: str | None = None, stream=None, out=None) -> np.ndarray:
        """Host buffers in, host f32 [B, H] out (``jb_encode_text``); ``out``
        may be a caller-owned (e.g. pinned) C-contiguous f32 [B, H] array."""
        ids = np.ascontiguousarray(ids, dtype=np.uint32)
        lens = np.ascontiguousarray(lens, dtype=np.uint32)
        B, S = ids.shape
        if out is None:
            out = np.empty((B, self.info.hidden), dtype=np.float32)
        elif (out.dtype != np.float32 or out.shape != (B, self.info.hidden)
              or not out.flags.c_contiguous):
            raise ValueError("out must be a C-contiguous float32 [batch, hidden] array")
        try:
            check(lib().jb_encode_text(self._h, _ptr(ids), _ptr(lens), B, S,
                                       POOLING[pooling or self.pooling], _ptr(out),
                                       _stream_ptr(stream)))
        except JbError as e:
            _raise_seq(e)
        return out

    def forward(self, input_ids, mask) -> np.ndarray:
        """``Bert::forward`` (bert.rs:279-282): pooled and L2-normalised."""
        return self.encode(input_ids, mask_to_lengths(mask))

    def encode_device(self, ids, lens, out, pooling: str | None = None, stream=None):
        """Device tensors (torch, uint32/int32 ids and lens, f32 out); async."""
        B, S = ids.shape
        try:
            check(lib().jb_encode_text_device(self._h, _ptr(ids), _ptr(lens), B, S,
                                              POOLING[pooling or self.pooling], _ptr(out),
                                              _stream_ptr(stream)))
        except JbError as e:
            _raise_seq(e)
        return out

    def forward_hidden(self, input_ids, mask):
        """``Bert::forward_hidden`` (bert.rs:257-276) -> torch f32 [B, S, H] on
        the model's device, zeros at padded positions."""
        import torch
        lens = mask_to_lengths(mask)
        dev = torch.device("cuda", self.device)
        ids_t = torch.from_numpy(np.ascontiguousarray(input_ids, dtype=np.int32)).to(dev)
        lens_t = torch.from_numpy(lens.astype(np.int32)).to(dev)
        B, S = ids_t.shape
        out = torch.empty((B, S, self.info.hidden), dtype=torch.float32, device=dev)
        stream = torch.cuda.current_stream(dev)
        try:
            check(lib().jb_forward_hidden_device(self._h, _ptr(ids_t), _ptr(lens_t), B, S,
                                                 _ptr(out), _stream_ptr(stream)))
        except JbError as e:
            _raise_seq(e)
        self.sync(stream)
        return out


class OpenClipVisionTransformer(Model):
    """OpenCLIP vision tower + ``l2_normalize`` on the B200 library."""
    FAMILY = L.FAMILY_CLIP_VISION

    def __init__(self, *a, **kw):
        super().__init__(*a, **kw)
        if self.info.family != L.FAMILY_CLIP_VISION:
            raise JbError(L.ERR_INVALID, "not an OpenCLIP vision checkpoint")

    def embed_dim(self) -> int:
        return self.info.output_dim

    def image_size(self) -> int:
        return self.info.image_size

    def forward_image(self, pixels, stream=None) -> np.ndarray:
        px = np.ascontiguousarray(pixels, dtype=np.float32)
        B = px.shape[0]
        out = np.zeros((B, self.info.output_dim), dtype=np.float32)
        check(lib().jb_encode_image(self._h, _ptr(px), B, _ptr(out), _stream_ptr(stream)))
        return out

    def encode_rgb8(self, images, stream=None) -> np.ndarray:
        """Decoded RGB8 images (``[h, w, 3]`` uint8 arrays of any sizes) ->
        host f32 [B, embed_dim]; padding, Catmull-Rom resize and normalisation
        run on the device (``jb_encode_image_rgb8``)."""
        buf, offs, ws, hs = pack_rgb8(images)
        out = np.zeros((len(images), self.info.output_dim), dtype=np.float32)
        check(lib().jb_encode_image_rgb8(self._h, buf.ctypes.data, buf.nbytes, offs.ctypes.data,
                                         ws.ctypes.data, hs.ctypes.data, len(images), _ptr(out),
                                         _stream_ptr(stream)))
        return out

    def forward_image_device(self, pixels, out, stream=None):
        check(lib().jb_encode_image_device(self._h, _ptr(pixels), pixels.shape[0], _ptr(out),
                                           _stream_ptr(stream)))
        return out


class OpenClipText(Model):
    """``jammi_encoders::ClipText`` (crates/jammi-encoders/src/clip_text.rs) on
    the B200 library: token ids -> L2-normalised ``[B, embed_dim]`` in the
    shared CLIP space, pooled at each row's EOT token (its largest id)."""
    FAMILY = L.FAMILY_CLIP_TEXT

    def __init__(self, *a, **kw):
        super().__init__(*a, **kw)
        if self.info.family != L.FAMILY_CLIP_TEXT:
            raise JbError(L.ERR_INVALID, "not an OpenCLIP text tower")

    def embed_dim(self) -> int:
        return self.info.output_dim

    def hidden_size(self) -> int:
        return self.info.hidden

    def context_length(self) -> int:
        return self.info.max_seq

    def encode(self, ids, stream=None) -> np.ndarray:
        """Host ids [B, S] (uint32) -> host f32 [B, embed_dim] (``jb_encode_text``;
        lengths and pooling do not apply)."""
        ids = np.ascontiguousarray(ids, dtype=np.uint32)
        B, S = ids.shape
        out = np.zeros((B, self.info.output_dim), dtype=np.float32)
        try:
            check(lib().jb_encode_text(self._h, _ptr(ids), None, B, S, L.POOL_MEAN, _ptr(out),
                                       _stream_ptr(stream)))
        except JbError as e:
            _raise_seq(e)
        return out

    def forward(self, input_ids, attention_mask=None) -> np.ndarray:
        """``ClipText::forward`` (clip_text.rs:296-331); the mask is accepted and
        unused, as there."""
        return self.encode(input_ids)

    def encode_device(self, ids, out, stream=None):
        """Device ids (torch int32/uint32 [B, S]) -> device f32 out; async."""
        B, S = ids.shape
        try:
            check(lib().jb_encode_text_device(self._h, _ptr(ids), None, B, S, L.POOL_MEAN,
                                              _ptr(out), _stream_ptr(stream)))
        except JbError as e:
            _raise_seq(e)
        return out


def pack_rgb8(images):
    """RGB8 ``[h, w, 3]`` arrays -> (bytes, int64 offsets, int32 widths, int32 heights)."""
    imgs = [np.ascontiguousarray(im, dtype=np.uint8) for im in images]
    for im in imgs:
        if im.ndim != 3 or im.shape[2] != 3:
            raise ValueError("images must be [h, w, 3] uint8 (RGB8)")
    sizes = [im.nbytes for im in imgs]
    offs = np.concatenate([[0], np.cumsum(sizes)[:-1]]).astype(np.int64) if imgs else np.zeros(0, np.int64)
    buf = np.concatenate([im.reshape(-1) for im in imgs]) if imgs else np.zeros(1, np.uint8)
    ws = np.array([im.shape[1] for im in imgs], dtype=np.int32)
    hs = np.array([im.shape[0] for im in imgs], dtype=np.int32)
    return buf, offs, ws, hs


POOLING_NAMES = {v: k for k, v in POOLING.items()}


def pooling_from_config(cfg=None) -> str:
    """The pooling a 1_Pooling/config.json declares (``jb_pooling_from_config``):
    ``cfg`` is the file's JSON text or parsed dict, None when there is no file."""
    import ctypes
    out = ctypes.c_int()
    text = None if cfg is None else (cfg if isinstance(cfg, str) else json.dumps(cfg)).encode()
    check(lib().jb_pooling_from_config(text, ctypes.byref(out)))
    return POOLING_NAMES[out.value]


def pooling_from_model_dir(model_dir: str) -> str:
    """``jb_pooling_from_model_dir``: <model_dir>/1_Pooling/config.json, mean if absent."""
    import ctypes
    out = ctypes.c_int()
    check(lib().jb_pooling_from_model_dir(str(model_dir).encode(), ctypes.byref(out)))
    return POOLING_NAMES[out.value]


def load_model(weights_path: str, config_path_or_dict, device: int = 0, fmt: str = "bf16",
               pooling: str | None = None, tower: str = "vision"):
    """``CandleBackend::load`` for the BERT and OpenCLIP arms: the family is
    detected from the config (``model_cfg`` -> OpenCLIP); an OpenCLIP checkpoint
    holds both towers, ``tower`` ("vision" or "text") picks one.  A text
    encoder's pooling defaults to what the checkpoint directory's
    1_Pooling/config.json declares (mean without one)."""
    cfg = config_path_or_dict
    if isinstance(cfg, str) and os.path.exists(cfg):
        cfg = json.load(open(cfg))
    if isinstance(cfg, str):
        cfg = json.loads(cfg)
    if "model_cfg" in cfg:
        if tower == "text":
            return OpenClipText(weights_path, cfg, device, fmt)
        return OpenClipVisionTransformer(weights_path, cfg, device, fmt)
    if pooling is None:
        pooling = pooling_from_model_dir(os.path.dirname(os.path.abspath(weights_path)))
    return Bert(weights_path, cfg, device, fmt, pooling=pooling)
