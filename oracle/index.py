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
