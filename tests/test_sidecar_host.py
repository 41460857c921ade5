"""CPU checks of the host side of jammi_b200.sidecar.SidecarIndex: the
_row_id map of the ok rows, the tie ranks it hands to the build (ascending
_row_id order, as SidecarIndex orders equal distances), the results named by
_row_id, and the bundle files save() writes (sidecar.rs:498-571).  The C
library is replaced by a stand-in that keeps its store in numpy and answers
through oracle/index.py, so these tests run without a GPU."""
import ctypes
import json
import struct

import numpy as np
import pytest

from oracle import index as oi


class FakeSidecarLib:
    """jb_sidecar_* over numpy: one handle, the oracle as the arithmetic."""

    def __init__(self):
        self.store = None
        self.dim = 0
        self.precision = 3
        self.rank = None
        self.tau = None

    @staticmethod
    def _arr(ptr, dtype, count):
        return np.ctypeslib.as_array(ctypes.cast(ptr, ctypes.POINTER(np.ctypeslib.as_ctypes_type(dtype))),
                                     shape=(count,))

    def jb_sidecar_create(self, device, dim, precision, out):
        self.dim, self.precision = dim, precision
        self.store = np.zeros((0, dim), np.float32)
        out._obj.value = 1
        return 0

    def jb_sidecar_add(self, h, vec, bits, rows, first, added):
        v = self._arr(vec, np.float32, rows * self.dim).reshape(rows, self.dim)
        b = None if not bits else self._arr(bits, np.uint8, (rows + 7) // 8)
        first._obj.value = len(self.store)
        kept = oi.sidecar_add(v, b)
        self.store = np.concatenate([self.store, kept])
        added._obj.value = len(kept)
        self.rank = None
        return 0

    def jb_sidecar_build(self, h, kind, rank):
        n = len(self.store)
        self.rank = None if not rank else self._arr(rank, np.uint32, n).astype(np.int64)
        if self.precision == 3 and n:
            self.tau = oi.fit_binary_threshold(self.store, "median" if kind == 1 else "mean")
        return 0

    def jb_sidecar_len(self, h):
        return len(self.store)

    def _answer(self, keys, dist, nq, k, got):
        self._arr(keys, np.int64, nq * k)[:] = got[0].reshape(-1)
        self._arr(dist, np.float32, nq * k)[:] = got[1].reshape(-1)

    def jb_sidecar_search(self, h, q, nq, k, keys, dist):
        queries = self._arr(q, np.float32, nq * self.dim).reshape(nq, self.dim)
        prec = "binary" if self.precision == 3 else "f32"
        self._answer(keys, dist, nq, k, oi.sidecar_search(self.store, queries, k, prec, self.tau, self.rank))
        return 0

    def jb_sidecar_search_final(self, h, q, nq, k, over, keys, dist):
        queries = self._arr(q, np.float32, nq * self.dim).reshape(nq, self.dim)
        prec = "binary" if self.precision == 3 else "f32"
        self._answer(keys, dist, nq, k, oi.search_final(self.store, queries, k, over, self.tau, prec, self.rank))
        return 0

    def jb_sidecar_export(self, h, exact, codes, tau):
        n = len(self.store)
        if exact:
            self._arr(exact, np.float32, n * self.dim)[:] = self.store.reshape(-1)
        if codes:
            c = oi.pack_threshold_bits(self.store, self.tau)
            self._arr(codes, np.uint8, c.size)[:] = c.reshape(-1)
        if tau:
            self._arr(tau, np.float32, self.dim)[:] = self.tau
        return 0

    def jb_sidecar_free(self, h):
        pass


@pytest.fixture
def fake(monkeypatch):
    import jammi_b200.sidecar as sc
    f = FakeSidecarLib()
    monkeypatch.setattr(sc, "lib", lambda: f)
    return f


def test_row_map_keeps_the_ok_rows_in_order(fake):
    from jammi_b200.sidecar import SidecarIndex
    idx = SidecarIndex(8, "binary")
    rng = np.random.default_rng(0)
    v = rng.standard_normal((10, 8)).astype(np.float32)
    ok = np.array([1, 0, 1, 1, 0, 0, 1, 1, 1, 0], bool)
    assert idx.write_batch(v, np.packbits(ok, bitorder="little"), [f"r{i}" for i in range(10)]) == 6
    assert idx.row_map == ["r0", "r2", "r3", "r6", "r7", "r8"]
    assert idx.row_index["r6"] == 3 and "r1" not in idx.row_index
    idx.add("z", v[1])
    assert idx.row_index["z"] == 6 and len(idx) == 7
    with pytest.raises(ValueError):
        idx.add("bad", np.zeros(7, np.float32))
    with pytest.raises(ValueError):
        idx.add_batch(["a"], v[:2])


def test_ties_follow_row_id_order(fake):
    """Equal distances come back in ascending _row_id order, not key order."""
    from jammi_b200.sidecar import SidecarIndex
    idx = SidecarIndex(4, "f32")
    ids = ["row-9", "row-10", "row-1", "row-2"]  # string order: row-1, row-10, row-2, row-9
    idx.add_batch(ids, np.tile(np.array([[1, 2, 3, 4]], np.float32), (4, 1)))
    idx.build()
    assert [rid for rid, _ in idx.search(np.array([1, 2, 3, 4], np.float32), 4)] == sorted(ids)
    with pytest.raises(ValueError):  # a repeated _row_id has no order
        idx.add("row-1", np.ones(4, np.float32))
        idx.build()


def test_finalize_and_search_final(fake):
    from jammi_b200.sidecar import SidecarIndex
    from test_index_oracle import splitmix_vector
    empty = SidecarIndex(64, "binary")
    assert empty.finalize() == (0, None)
    assert empty.search(np.ones(64, np.float32), 3) == []
    idx = SidecarIndex(64, "binary")
    rows = np.stack([splitmix_vector(i + 100, 64) for i in range(24)])
    idx.add_batch([f"row-{i}" for i in range(24)], rows)
    n, built = idx.finalize()
    assert n == 24 and built is idx and idx.threshold_kind == "median"
    q = (rows[9] + np.float32(0.05) * splitmix_vector(999, 64)).astype(np.float32)
    assert idx.search_final(q, 5, 32)[0][0] == "row-9"


def test_save_writes_the_bundle_files(fake, tmp_path):
    from jammi_b200.sidecar import SidecarIndex
    idx = SidecarIndex(16, "binary")
    rng = np.random.default_rng(1)
    v = rng.standard_normal((5, 16)).astype(np.float32)
    idx.add_batch(["a", "bb", "ccc", "dddd", "é"], v)
    idx.build("mean")
    idx.save(str(tmp_path / "emb"))
    raw = (tmp_path / "emb.rowmap").read_bytes()
    assert struct.unpack_from("<I", raw, 0)[0] == 1
    off, got = 4, []
    while off < len(raw):
        (n,) = struct.unpack_from("<I", raw, off)
        got.append(raw[off + 4:off + 4 + n].decode("utf-8"))
        off += 4 + n
    assert got == ["a", "bb", "ccc", "dddd", "é"]
    assert np.array_equal(np.fromfile(tmp_path / "emb.rawf32", np.float32).reshape(5, 16), v)
    tau = oi.fit_binary_threshold(v, "mean")
    assert np.array_equal(np.fromfile(tmp_path / "emb.threshold", np.float32), tau)
    assert np.array_equal(np.fromfile(tmp_path / "emb.codes", np.uint8).reshape(5, 2), oi.pack_threshold_bits(v, tau))
    man = json.loads((tmp_path / "emb.manifest.json").read_text())
    assert man["version"] == 3 and man["dimensions"] == 16 and man["count"] == 5
    assert man["metric"] == "hamming" and man["scalar_kind"] == "binary"
    assert man["binary_threshold_kind"] == "mean"
