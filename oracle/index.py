"""CPU oracle for the vector side of the reference's index module (test
oracle only: tests and the checker import it, the library never does).

* ``fit_binary_threshold`` -- fit_binary_threshold / mean_threshold /
  median_threshold, crates/jammi-db/src/index/sidecar.rs:162-216: over the
  first min(rows, 100000) rows, the per-dimension mean (an f64 sum in row
  order, divided by the row count, cast to f32) or median (f32 total order,
  the two central values averaged in f32 for an even count); zeros without
  rows.
* ``pack_threshold_bits`` -- sidecar.rs:232-241: bit i = v[i] > tau[i],
  LSB-first, ceil(dim / 8) bytes, padding bits 0.
* ``cosine_distances`` -- cosine_distance, crates/jammi-numerics/src/
  distance.rs:6-21: the dot product and both squared norms accumulate in
  f32 in dimension order (each product and each sum rounded to f32, no fused
  multiply-add), denominator sqrt(|a|^2) * sqrt(|b|^2), distance 1 when the
  denominator is below f32 epsilon, else 1 - dot / denominator.
* ``exact_search`` -- exact_vector_search, crates/jammi-db/src/index/
  exact.rs:119-175: the k smallest distances, ties broken by ascending
  _row_id (here: a caller-given rank per row, row order by default).
* ``sidecar_add`` -- ResultSink::write_batch (crates/jammi-ai/src/pipeline/
  result_sink.rs:61-83) feeding SidecarIndex::add (sidecar.rs:754-790): the
  rows whose validity bit is set, in row order, one key each.
* ``hamming_distances`` / ``sidecar_search`` -- SidecarIndex::search
  (sidecar.rs:826-864): a Binary sidecar compares the query's threshold code
  with every key's code by differing bits (usearch's Hamming metric over
  b1x8); an F32 one by cosine distance.  The k nearest under (distance,
  rank), scanning every key (the reference's HNSW graph approximates this).
* ``search_final`` -- SegmentedIndex::search_final (crates/jammi-db/src/
  index/segment.rs:239-264): k x oversample (at least k) candidates by
  search, each rescored by cosine distance to its exact vector, ordered by
  (distance under f32::total_cmp, rank), truncated to k.
"""
from __future__ import annotations

import numpy as np

SAMPLE_CAP = 100_000
F32_EPS = np.float32(np.finfo(np.float32).eps)


def total_keys(x: np.ndarray) -> np.ndarray:
    """f32 -> uint32 keys whose unsigned order is f32::total_cmp's order."""
    b = np.ascontiguousarray(x, np.float32).view(np.uint32)
    return np.where(b & np.uint32(0x80000000), ~b, b | np.uint32(0x80000000)).astype(np.uint32)


def from_total_keys(k: np.ndarray) -> np.ndarray:
    k = np.asarray(k, np.uint32)
    b = np.where(k & np.uint32(0x80000000), k & np.uint32(0x7FFFFFFF), ~k).astype(np.uint32)
    return b.view(np.float32)


def fit_binary_threshold(v: np.ndarray, kind: str = "median") -> np.ndarray:
    v = np.asarray(v, np.float32)
    rows, dim = v.shape
    n = min(rows, SAMPLE_CAP)
    if dim == 0:
        return np.zeros(0, np.float32)
    if kind == "mean":
        s = np.cumsum(v[:n].astype(np.float64), axis=0)[-1] if n else np.zeros(dim)
        return (s / float(max(n, 1))).astype(np.float32)
    if n == 0:
        return np.zeros(dim, np.float32)
    col = from_total_keys(np.sort(total_keys(v[:n]), axis=0))
    mid = n // 2
    if n % 2 == 0:
        return ((col[mid - 1] + col[mid]) / np.float32(2.0)).astype(np.float32)
    return col[mid].copy()


def pack_threshold_bits(v: np.ndarray, tau: np.ndarray) -> np.ndarray:
    v = np.atleast_2d(np.asarray(v, np.float32))
    return np.packbits(v > np.asarray(tau, np.float32)[None, :], axis=1, bitorder="little")


def cosine_distances(query: np.ndarray, corpus: np.ndarray) -> np.ndarray:
    q = np.asarray(query, np.float32)
    c = np.asarray(corpus, np.float32)
    n = c.shape[0]
    dot = np.zeros(n, np.float32)
    nb = np.zeros(n, np.float32)
    na = np.float32(0.0)
    for i in range(q.shape[0]):
        a, b = q[i], c[:, i]
        dot = (dot + (a * b).astype(np.float32)).astype(np.float32)
        nb = (nb + (b * b).astype(np.float32)).astype(np.float32)
        na = np.float32(na + np.float32(a * a))
    denom = (np.sqrt(na).astype(np.float32) * np.sqrt(nb)).astype(np.float32)
    with np.errstate(divide="ignore", invalid="ignore"):
        dist = (np.float32(1.0) - (dot / denom).astype(np.float32)).astype(np.float32)
    return np.where(denom < F32_EPS, np.float32(1.0), dist).astype(np.float32)


def exact_search(corpus: np.ndarray, queries: np.ndarray, k: int, tie_rank=None):
    """(idx int64 [q, min(k, n)], dist f32 [q, min(k, n)]), ascending
    (distance, rank)."""
    corpus = np.asarray(corpus, np.float32)
    n = corpus.shape[0]
    rank = np.arange(n, dtype=np.int64) if tie_rank is None else np.asarray(tie_rank, np.int64)
    kk = min(k, n)
    idx = np.zeros((len(queries), kk), np.int64)
    dist = np.zeros((len(queries), kk), np.float32)
    for j, q in enumerate(np.asarray(queries, np.float32)):
        d = cosine_distances(q, corpus)
        order = np.lexsort((rank, d + np.float32(0.0)))[:kk]  # -0 sorts as +0, NaN last
        idx[j], dist[j] = order, d[order]
    return idx, dist


def cosine_distance_loop(a, b) -> np.float32:
    """distance.rs:6-21 as a scalar loop (pins the vectorised form)."""
    dot = na = nb = np.float32(0.0)
    for x, y in zip(np.asarray(a, np.float32), np.asarray(b, np.float32)):
        dot = np.float32(dot + np.float32(x * y))
        na = np.float32(na + np.float32(x * x))
        nb = np.float32(nb + np.float32(y * y))
    denom = np.float32(np.sqrt(na) * np.sqrt(nb))
    if denom < F32_EPS:
        return np.float32(1.0)
    return np.float32(np.float32(1.0) - np.float32(dot / denom))


def sidecar_add(vectors: np.ndarray, validity=None) -> np.ndarray:
    """The rows of ``vectors`` [rows, dim] whose bit in the LSB-first
    ``validity`` bitmap is set (None = all), in row order."""
    v = np.asarray(vectors, np.float32)
    if validity is None:
        return v.copy()
    bits = np.unpackbits(np.asarray(validity, np.uint8), bitorder="little")[: v.shape[0]].astype(bool)
    return v[bits]


def hamming_distances(qcode: np.ndarray, codes: np.ndarray) -> np.ndarray:
    """Differing bits of one packed query code and every packed row code."""
    x = np.bitwise_xor(np.asarray(codes, np.uint8), np.asarray(qcode, np.uint8)[None, :])
    return np.unpackbits(x, axis=1).sum(axis=1).astype(np.float32)


def _order(dist: np.ndarray, rank: np.ndarray, kk: int, total_order: bool) -> np.ndarray:
    key = total_keys(dist) if total_order else total_keys(dist + np.float32(0.0))
    return np.lexsort((rank, key))[:kk]


def sidecar_search(store: np.ndarray, queries: np.ndarray, k: int, precision: str = "binary",
                   tau=None, tie_rank=None):
    """(keys int64 [q, k], dist f32 [q, k]) with -1 / +inf past the store's
    length.  ``store`` is the exact f32 vectors in key order."""
    store = np.asarray(store, np.float32)
    n = store.shape[0]
    rank = np.arange(n, dtype=np.int64) if tie_rank is None else np.asarray(tie_rank, np.int64)
    keys = np.full((len(queries), k), -1, np.int64)
    dist = np.full((len(queries), k), np.inf, np.float32)
    kk = min(k, n)
    if kk == 0:
        return keys, dist
    codes = pack_threshold_bits(store, tau) if precision == "binary" else None
    for j, q in enumerate(np.asarray(queries, np.float32)):
        if precision == "binary":
            d = hamming_distances(pack_threshold_bits(q[None, :], tau)[0], codes)
        else:
            d = cosine_distances(q, store)
        o = _order(d, rank, kk, total_order=False)
        keys[j, :kk], dist[j, :kk] = o, d[o]
    return keys, dist


def search_final(store: np.ndarray, queries: np.ndarray, k: int, oversample: int, tau=None,
                 precision: str = "binary", tie_rank=None):
    """segment.rs:239-264 over one segment: an exact (F32) store answers as
    its search; a Binary one retrieves candidate_k = max(k * oversample, k)
    by Hamming distance, rescores by cosine distance and keeps k."""
    if precision != "binary":
        return sidecar_search(store, queries, k, precision, tau, tie_rank)
    store = np.asarray(store, np.float32)
    n = store.shape[0]
    rank = np.arange(n, dtype=np.int64) if tie_rank is None else np.asarray(tie_rank, np.int64)
    ck = max(k * max(oversample, 1), k)
    cand, _ = sidecar_search(store, queries, ck, "binary", tau, tie_rank)
    keys = np.full((len(queries), k), -1, np.int64)
    dist = np.full((len(queries), k), np.inf, np.float32)
    for j, q in enumerate(np.asarray(queries, np.float32)):
        c = cand[j][cand[j] >= 0]
        if len(c) == 0:
            continue
        d = cosine_distances(q, store[c])
        o = _order(d, rank[c], min(k, len(c)), total_order=True)
        keys[j, :len(o)], dist[j, :len(o)] = c[o], d[o]
    return keys, dist
