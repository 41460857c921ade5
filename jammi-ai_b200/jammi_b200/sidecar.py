"""SidecarIndex on the device: the reference's ANN sidecar
(crates/jammi-db/src/index/sidecar.rs:317-864) with its vector store, threshold
fit, sign-packing and search in libjammi_b200.so (``jb_sidecar_*``), and the
_row_id map, tie order and bundle files here.

``add_batch`` takes a job's output as ``jb_generate_embeddings`` leaves it --
f32 values [rows, dim] plus the LSB-first validity bitmap -- and keeps the ok
rows in row order, as ResultSink::write_batch (crates/jammi-ai/src/pipeline/
result_sink.rs:61-83) does before it calls SidecarIndex::add per row.
``finalize`` is ResultSink::finalize (result_sink.rs:85-96): build when any
row was added.
"""
from __future__ import annotations

import ctypes
import json
import os
import struct

import numpy as np

from ._lib import check, lib

ROWMAP_VERSION = 1          # sidecar.rs:11
ANN_MANIFEST_VERSION = 3    # sidecar.rs:35
PRECISIONS = {"f32": 0, "binary": 3}
THRESHOLD_KINDS = {"mean": 0, "median": 1}
DEFAULT_THRESHOLD_KIND = "median"   # DEFAULT_BINARY_THRESHOLD_KIND, sidecar.rs:141
DEFAULT_BINARY_OVERSAMPLE = 32      # StoragePrecision::default_oversample, config.rs:503-508
MAX_CANDIDATES = 1024


def _ptr(a) -> int:
    """Address of a numpy array (host) or a torch tensor (host or device)."""
    if a is None:
        return 0
    if isinstance(a, np.ndarray):
        return a.ctypes.data
    return a.data_ptr()


def _f32(a):
    """A contiguous f32 numpy array, or a contiguous f32 torch tensor as is."""
    if isinstance(a, np.ndarray) or not hasattr(a, "data_ptr"):
        return np.ascontiguousarray(a, np.float32)
    if str(a.dtype) != "torch.float32" or not a.is_contiguous():
        raise ValueError("torch vectors must be contiguous float32")
    return a


class SidecarIndex:
    """One device's sidecar: ``SidecarIndex::new(dimensions, ann, precision)``
    with precision "f32" or "binary"."""

    def __init__(self, dimensions: int, precision: str = "binary", device: int = 0):
        if precision not in PRECISIONS:
            raise ValueError(f"precision must be one of {sorted(PRECISIONS)}")
        self.dimensions = int(dimensions)
        self.precision = precision
        self.device = device
        self.row_map: list[str] = []
        self.row_index: dict[str, int] = {}
        self.threshold_kind: str | None = None
        self._built = False
        h = ctypes.c_void_p()
        check(lib().jb_sidecar_create(device, self.dimensions, PRECISIONS[precision], ctypes.byref(h)))
        self._h = h

    # -- insert -------------------------------------------------------------
    def add(self, row_id: str, vector) -> None:
        """``SidecarIndex::add``: one vector under the next key."""
        v = np.asarray(vector, np.float32).reshape(-1)
        if v.shape[0] != self.dimensions:
            raise ValueError(f"Vector dimension mismatch: expected {self.dimensions}, got {v.shape[0]}")
        self.add_batch([row_id], v[None, :])

    def add_batch(self, row_ids, vectors, validity=None) -> int:
        """Append the rows of ``vectors`` [rows, dim] whose validity bit is
        set (all when None), in row order; ``row_ids`` names every row of the
        batch.  Returns how many rows were taken."""
        v = _f32(vectors)
        rows = int(v.shape[0])
        if rows and int(v.shape[1]) != self.dimensions:
            raise ValueError(f"Vector dimension mismatch: expected {self.dimensions}, got {int(v.shape[1])}")
        row_ids = list(row_ids)
        if len(row_ids) != rows:
            raise ValueError("one row id per row")
        bits = None
        if validity is not None:
            bits = np.ascontiguousarray(validity, np.uint8) if isinstance(validity, np.ndarray) or \
                not hasattr(validity, "data_ptr") else validity
            if int(bits.shape[0]) * 8 < rows:
                raise ValueError("validity bitmap shorter than the batch")
        first = ctypes.c_int64()
        added = ctypes.c_int64()
        check(lib().jb_sidecar_add(self._h, _ptr(v), _ptr(bits), rows, ctypes.byref(first), ctypes.byref(added)))
        if bits is None:
            kept = row_ids
        else:
            mask = np.unpackbits(np.asarray(bits.cpu() if hasattr(bits, "cpu") else bits, np.uint8),
                                 bitorder="little")[:rows].astype(bool)
            kept = [rid for rid, ok in zip(row_ids, mask) if ok]
        if len(kept) != added.value:
            raise RuntimeError("sidecar add: device and host disagree on the valid row count")
        key = first.value
        for rid in kept:
            self.row_index[rid] = key
            self.row_map.append(rid)
            key += 1
        if kept:
            self._built = False
        return added.value

    def write_batch(self, values, validity, row_ids) -> int:
        """ResultSink::write_batch over a job's output (values, validity bitmap)."""
        return self.add_batch(row_ids, values, validity)

    def build(self, threshold_kind: str = DEFAULT_THRESHOLD_KIND) -> None:
        """``SidecarIndex::build``: fit tau and pack every key (Binary); equal
        distances then rank by ascending _row_id."""
        if threshold_kind not in THRESHOLD_KINDS:
            raise ValueError(f"threshold kind must be one of {sorted(THRESHOLD_KINDS)}")
        rank = None
        if self.row_map:
            order = sorted(range(len(self.row_map)), key=self.row_map.__getitem__)
            rank = np.empty(len(order), np.uint32)
            rank[np.asarray(order, np.int64)] = np.arange(len(order), dtype=np.uint32)
            if len(self.row_index) != len(self.row_map):
                raise ValueError("repeated _row_id in the sidecar")
        check(lib().jb_sidecar_build(self._h, THRESHOLD_KINDS[threshold_kind], _ptr(rank)))
        if self.precision == "binary" and self.row_map:
            self.threshold_kind = threshold_kind
        self._built = True

    def finalize(self):
        """ResultSink::finalize: build when at least one row was added;
        returns (row count, self or None)."""
        if not self.row_map:
            return 0, None
        self.build()
        return len(self.row_map), self

    def __len__(self) -> int:
        return int(lib().jb_sidecar_len(self._h))

    # -- search -------------------------------------------------------------
    def _queries(self, queries):
        q = _f32(queries)
        if q.ndim == 1:
            q = q.reshape(1, -1)
        if int(q.shape[1]) != self.dimensions:
            raise ValueError(f"query dimension mismatch: expected {self.dimensions}, got {int(q.shape[1])}")
        return q

    def search_keys(self, queries, k: int):
        """keys int64 / dist f32 [n_queries, k] (-1 / +inf past len)."""
        q = self._queries(queries)
        nq = int(q.shape[0])
        keys = np.empty((nq, k), np.int64)
        dist = np.empty((nq, k), np.float32)
        check(lib().jb_sidecar_search(self._h, _ptr(q), nq, k, _ptr(keys), _ptr(dist)))
        return keys, dist

    def search_final_keys(self, queries, k: int, oversample: int = DEFAULT_BINARY_OVERSAMPLE):
        q = self._queries(queries)
        nq = int(q.shape[0])
        keys = np.empty((nq, k), np.int64)
        dist = np.empty((nq, k), np.float32)
        check(lib().jb_sidecar_search_final(self._h, _ptr(q), nq, k, oversample, _ptr(keys), _ptr(dist)))
        return keys, dist

    def _named(self, keys, dist):
        return [(self.row_map[int(i)], float(d)) for i, d in zip(keys, dist) if i >= 0]

    def search(self, query, k: int):
        """``SidecarIndex::search`` for one query: [(row_id, distance)]."""
        if not self.row_map:
            return []
        keys, dist = self.search_keys(query, min(k, len(self.row_map)))
        return self._named(keys[0], dist[0])

    def search_final(self, query, k: int, oversample: int = DEFAULT_BINARY_OVERSAMPLE):
        """``SegmentedIndex::search_final`` for one query (one segment)."""
        if not self.row_map:
            return []
        keys, dist = self.search_final_keys(query, k, oversample)
        return self._named(keys[0], dist[0])

    # -- vectors and files --------------------------------------------------
    def exact_vectors(self) -> np.ndarray:
        out = np.empty((len(self.row_map), self.dimensions), np.float32)
        check(lib().jb_sidecar_export(self._h, _ptr(out), None, None))
        return out

    def codes(self) -> np.ndarray:
        """Per key, the packed threshold code a usearch b1x8 graph is given."""
        out = np.empty((len(self.row_map), (self.dimensions + 7) // 8), np.uint8)
        check(lib().jb_sidecar_export(self._h, None, _ptr(out), None))
        return out

    def threshold(self) -> np.ndarray:
        out = np.empty(self.dimensions, np.float32)
        check(lib().jb_sidecar_export(self._h, None, None, _ptr(out)))
        return out

    def get_exact(self, row_id: str):
        key = self.row_index.get(row_id)
        if key is None:
            return None
        return self.exact_vectors()[key]

    def save(self, base_path: str) -> None:
        """The bundle's files beside ``base_path`` (SidecarIndex::save,
        sidecar.rs:498-571): .rowmap (u32 LE version, then per key a u32 LE
        byte length and the UTF-8 _row_id), .rawf32 (Binary: exact vectors in
        key order), .threshold (Binary: tau as f32), .codes (Binary: the
        packed code of every key -- what the graph library is given; the
        graph itself is the library's) and .manifest.json."""
        base = os.path.splitext(base_path)[0]
        with open(base + ".rowmap", "wb") as f:
            f.write(struct.pack("<I", ROWMAP_VERSION))
            for rid in self.row_map:
                b = rid.encode("utf-8")
                f.write(struct.pack("<I", len(b)))
                f.write(b)
        files = {"rowmap": os.path.basename(base + ".rowmap")}
        if self.precision == "binary" and self.row_map:
            self.exact_vectors().tofile(base + ".rawf32")
            if self._built:
                self.threshold().tofile(base + ".threshold")
                self.codes().tofile(base + ".codes")
                files["codes"] = os.path.basename(base + ".codes")
        manifest = {
            "version": ANN_MANIFEST_VERSION,
            "dimensions": self.dimensions,
            "count": len(self.row_map),
            "metric": "hamming" if self.precision == "binary" else "cosine",
            "backend": "jammi_b200",
            "scalar_kind": self.precision,
            "binary_threshold_kind": self.threshold_kind,
            "files": files,
        }
        with open(base + ".manifest.json", "w") as f:
            json.dump(manifest, f, indent=2)

    def close(self) -> None:
        if getattr(self, "_h", None) and self._h.value:
            lib().jb_sidecar_free(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


__all__ = ["SidecarIndex"]
