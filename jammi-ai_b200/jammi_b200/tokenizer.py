"""``Tokenizer``: the library's host-side tokenizers (``jb_tokenizer_*``), the
counterpart of the reference's ``TokenizerWrapper`` (crates/jammi-ai/src/model/
tokenizer.rs): a model's tokenizer.json (WordPiece or BPE, byte-level or
character-level) or OpenCLIP's merges file (clip_bpe.rs).

Calling it on a list of texts returns one uint32 id array per text, so it can
be handed to ``driver.embed_texts`` as the ``tokenize`` callable."""
from __future__ import annotations

import ctypes

import numpy as np

from . import _lib as L
from ._lib import check, lib


class Tokenizer:
    """``Tokenizer(tokenizer_json)``: a model's tokenizer.json;
    ``Tokenizer.clip_bpe(path)``: the OpenCLIP text tower's BPE from its merges
    file.  ``max_length`` 0 applies the file's own truncation, if any."""

    def __init__(self, tokenizer_json: str | None = None, max_length: int = 0, _handle=None):
        if _handle is None:
            h = ctypes.c_void_p()
            check(lib().jb_tokenizer_load(str(tokenizer_json).encode(), ctypes.byref(h)))
            _handle = h
        self._h = _handle
        self.max_length = int(max_length)

    @classmethod
    def clip_bpe(cls, merges_path: str, max_length: int = 0):
        h = ctypes.c_void_p()
        check(lib().jb_tokenizer_load_clip_bpe(str(merges_path).encode(), ctypes.byref(h)))
        return cls(max_length=max_length, _handle=h)

    def close(self):
        if getattr(self, "_h", None):
            lib().jb_tokenizer_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def encode_ragged(self, texts, max_length: int | None = None, null_rows: bool = False):
        """texts -> (ids uint32, offsets uint64 [n + 1]), the layout of
        ``driver.generate_embeddings``.  ``null_rows``: a None or empty text is
        a row without tokens (``jb_tokenize_rows``, the embedding path's row
        rule) instead of the encoding of the empty string."""
        enc = [b"" if t is None else t.encode("utf-8") for t in texts]
        fn = lib().jb_tokenize_rows if null_rows else lib().jb_tokenize
        n = len(enc)
        ptrs = (ctypes.c_char_p * max(n, 1))(*enc)
        sizes = np.array([len(e) for e in enc], dtype=np.uint64)
        offsets = np.zeros(n + 1, dtype=np.uint64)
        ml = self.max_length if max_length is None else int(max_length)
        # One pass in the common case: a token covers at least one byte, so
        # bytes + a few ids per text (specials, a prefix space) bound the
        # output; a text dense in added tokens may need the exact-size retry.
        cap = int(sizes.sum()) + 4 * n + 64
        ids = np.empty(cap, dtype=np.uint32)
        st = fn(self._h, ctypes.cast(ptrs, ctypes.c_void_p), sizes.ctypes.data, n, ml,
                ids.ctypes.data, cap, offsets.ctypes.data)
        if st != L.OK and int(offsets[-1]) > cap:
            ids = np.empty(int(offsets[-1]), dtype=np.uint32)
            st = fn(self._h, ctypes.cast(ptrs, ctypes.c_void_p), sizes.ctypes.data, n, ml,
                    ids.ctypes.data, ids.size, offsets.ctypes.data)
        check(st)
        return ids[: int(offsets[-1])], offsets

    def __call__(self, texts, max_length: int | None = None):
        ids, offsets = self.encode_ragged(list(texts), max_length)
        return [ids[offsets[i]:offsets[i + 1]] for i in range(len(offsets) - 1)]
