"""GPU parity of the index-side ops (binary threshold fit, threshold
sign-packing, exact cosine search) against oracle/index.py, through the C
ABI on seeded inputs.  Every check is bit-exact: the threshold mean and the
distances follow the reference's f32/f64 operation order, the median and
the packing are exact by construction, and the top-k order is total."""
import numpy as np
import pytest

from oracle import index as oi

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")


def _ops():
    from jammi_b200 import ops
    return ops


def _bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def _vectors(rng, rows, dim):
    v = rng.standard_normal((rows, dim)).astype(np.float32)
    v[rng.random((rows, dim)) < 0.05] = 0.25  # repeated values
    if rows > 2:
        v[0] = -0.0
        v[1] = 0.0
    return v


@pytest.mark.parametrize("kind", ["mean", "median"])
@pytest.mark.parametrize("rows,dim", [(1, 5), (2, 33), (1000, 768), (4097, 100), (6001, 768)])
def test_fit_binary_threshold_bit_exact(dev, kind, rows, dim):
    rng = np.random.default_rng(rows * 7 + dim)
    v = _vectors(rng, rows, dim)
    got = _ops().fit_binary_threshold(torch.from_numpy(v).to(dev), kind).cpu().numpy()
    assert np.array_equal(_bits(got), _bits(oi.fit_binary_threshold(v, kind)))


@pytest.mark.parametrize("kind", ["mean", "median"])
def test_fit_binary_threshold_sample_cap(dev, kind):
    """Only the first 100000 rows are read (sidecar.rs:144-171)."""
    rng = np.random.default_rng(5)
    v = _vectors(rng, oi.SAMPLE_CAP + 3, 40)
    v[oi.SAMPLE_CAP:] = 1e30
    got = _ops().fit_binary_threshold(torch.from_numpy(v).to(dev), kind).cpu().numpy()
    assert np.array_equal(_bits(got), _bits(oi.fit_binary_threshold(v, kind)))
    assert np.all(np.abs(got) < 1e3)


def test_fit_binary_threshold_without_rows(dev):
    got = _ops().fit_binary_threshold(torch.zeros((0, 9), device=dev), "median").cpu().numpy()
    assert got.tolist() == [0.0] * 9


@pytest.mark.parametrize("rows,dim", [(1, 9), (3, 4), (1000, 768), (17, 1001)])
def test_pack_threshold_bits_bit_exact(dev, rows, dim):
    rng = np.random.default_rng(rows + dim)
    v = _vectors(rng, rows, dim)
    tau = oi.fit_binary_threshold(v, "median")
    got = _ops().pack_threshold_bits(torch.from_numpy(v).to(dev), torch.from_numpy(tau).to(dev)).cpu().numpy()
    assert np.array_equal(got, oi.pack_threshold_bits(v, tau))


def test_pack_threshold_bits_known_answer(dev):
    v = torch.tensor([[1.0, -1.0, 0.0, 2.0, -0.5, 0.5, -3.0, 4.0, 0.1]], device=dev)
    got = _ops().pack_threshold_bits(v, torch.zeros(9, device=dev)).cpu().numpy()
    assert got[0].tolist() == [0b1010_1001, 0b0000_0001]


@pytest.mark.parametrize("n,dim,nq,k", [(5000, 384, 19, 10), (1000, 768, 8, 1), (300, 33, 3, 100),
                                        (7, 16, 2, 10), (4096, 64, 9, 1024)])
def test_exact_search_bit_exact(dev, n, dim, nq, k):
    rng = np.random.default_rng(n + dim + nq + k)
    corpus = rng.standard_normal((n, dim)).astype(np.float32)
    corpus[::50] = corpus[0]  # equal distances: the tie rank decides
    corpus[1 % n] = 0.0       # zero magnitude: distance 1
    queries = rng.standard_normal((nq, dim)).astype(np.float32)
    queries[0] = corpus[min(5, n - 1)]
    rank = rng.permutation(n).astype(np.int32)
    ops = _ops()
    C, Q = torch.from_numpy(corpus).to(dev), torch.from_numpy(queries).to(dev)
    for tr in (None, rank):
        idx, dist = ops.exact_search(C, Q, k, tie_rank=None if tr is None else torch.from_numpy(tr).to(dev))
        want_idx, want_dist = oi.exact_search(corpus, queries, k, tr)
        assert np.array_equal(idx.cpu().numpy(), want_idx)
        assert np.array_equal(_bits(dist.cpu().numpy()), _bits(want_dist))


def test_exact_search_known_answer(dev):
    """crates/jammi-db/tests/it/index.rs:169-245: near, mid, far, opp."""
    corpus = torch.tensor([[0, 1, 0, 0], [1, 0, 0, 0], [0.7, 0.7, 0, 0], [-1, 0, 0, 0]],
                          dtype=torch.float32, device=dev)
    idx, dist = _ops().exact_search(corpus, torch.tensor([[1.0, 0, 0, 0]], device=dev), 4)
    assert idx.cpu().tolist() == [[1, 2, 0, 3]]
    assert dist.cpu().tolist()[0][0] == 0.0 and dist.cpu().tolist()[0][3] == 2.0


def test_exact_search_rejects_repeated_tie_ranks(dev):
    from jammi_b200._lib import JbError
    corpus = torch.ones((64, 8), device=dev)
    with pytest.raises(JbError):
        _ops().exact_search(corpus, corpus[:1].clone(), 5,
                            tie_rank=torch.zeros(64, dtype=torch.int32, device=dev))
    # the flag is cleared: the next search runs clean
    idx, _ = _ops().exact_search(corpus, corpus[:1].clone(), 5)
    assert idx.cpu().tolist() == [[0, 1, 2, 3, 4]]


def test_exact_search_rejects_repeated_tie_ranks_inside_k(dev):
    """Equal distances with equal ranks inside the k best have no order: an
    error, and every output slot is still written (no stale values)."""
    from jammi_b200._lib import JbError
    corpus = torch.ones((3, 8), device=dev)
    with pytest.raises(JbError):
        _ops().exact_search(corpus, corpus[:1].clone(), 3,
                            tie_rank=torch.zeros(3, dtype=torch.int32, device=dev))


# ---- device-resident sidecar (jb_sidecar_*): insert, build, search ---------

def _sidecar(dim, precision="binary"):
    from jammi_b200.sidecar import SidecarIndex
    return SidecarIndex(dim, precision, device=0)


def _string_rank(ids):
    order = sorted(range(len(ids)), key=ids.__getitem__)
    rank = np.empty(len(ids), np.int64)
    rank[order] = np.arange(len(ids))
    return rank


def _corpus(rng, rows, dim):
    v = rng.standard_normal((rows, dim)).astype(np.float32)
    v[::37] = v[0]  # repeated vectors: equal distances, the _row_id rank decides
    return v


@pytest.mark.parametrize("rows,dim", [(30000, 768), (1000, 37), (1, 5), (300, 100)])
def test_sidecar_add_keeps_valid_rows_in_order(dev, rows, dim):
    """write_batch + add: the ok rows of each batch, in row order, one key
    each; several batches (the first 30000-row case crosses the add staging
    chunk) accumulate; host numpy and device torch inputs alike."""
    rng = np.random.default_rng(rows + dim)
    v = _corpus(rng, rows, dim)
    ok = rng.random(rows) < 0.8
    bits = np.packbits(ok, bitorder="little")
    sc = _sidecar(dim)
    n1 = sc.add_batch([f"a{i}" for i in range(rows)], v, bits)
    n2 = sc.add_batch([f"b{i}" for i in range(rows)], torch.from_numpy(v).to(dev), torch.from_numpy(bits).to(dev))
    n3 = sc.add_batch([f"c{i}" for i in range(rows)], v)  # no bitmap: every row
    want = np.concatenate([oi.sidecar_add(v, bits), oi.sidecar_add(v, bits), v])
    assert (n1, n2, n3) == (int(ok.sum()), int(ok.sum()), rows)
    assert len(sc) == len(want) == len(sc.row_map)
    assert np.array_equal(_bits(sc.exact_vectors()), _bits(want))
    assert sc.row_index[f"c{rows - 1}"] == len(want) - 1
    sc.close()


@pytest.mark.parametrize("kind", ["median", "mean"])
@pytest.mark.parametrize("rows,dim", [(5000, 768), (777, 100), (3, 9)])
def test_sidecar_build_codes_and_threshold_bit_exact(dev, kind, rows, dim):
    rng = np.random.default_rng(rows * 3 + dim)
    v = _corpus(rng, rows, dim)
    sc = _sidecar(dim)
    sc.add_batch([str(i) for i in range(rows)], v)
    sc.build(kind)
    tau = oi.fit_binary_threshold(v, kind)
    assert np.array_equal(_bits(sc.threshold()), _bits(tau))
    assert np.array_equal(sc.codes(), oi.pack_threshold_bits(v, tau))
    sc.close()


@pytest.mark.parametrize("precision", ["binary", "f32"])
@pytest.mark.parametrize("rows,dim,nq,k", [(20000, 768, 11, 10), (900, 100, 5, 64), (50, 64, 3, 60)])
def test_sidecar_search_bit_exact(dev, precision, rows, dim, nq, k):
    """SidecarIndex::search: Hamming (Binary) or cosine (F32) distance to
    every key, ties by _row_id rank; keys and distances bit-exact."""
    rng = np.random.default_rng(rows + nq + k)
    v = _corpus(rng, rows, dim)
    ids = [f"row-{i}" for i in range(rows)]
    sc = _sidecar(dim, precision)
    sc.add_batch(ids, v)
    sc.build()
    q = rng.standard_normal((nq, dim)).astype(np.float32)
    q[0] = v[3]
    keys, dist = sc.search_keys(q, k)
    tau = oi.fit_binary_threshold(v, "median")
    wk, wd = oi.sidecar_search(v, q, k, precision, tau, _string_rank(ids))
    assert np.array_equal(keys, wk)
    assert np.array_equal(_bits(dist), _bits(wd))
    sc.close()


@pytest.mark.parametrize("rows,dim,nq,k,over", [(20000, 768, 7, 10, 32), (2000, 100, 4, 3, 300),
                                                (40, 64, 2, 8, 32), (5, 64, 1, 3, 0)])
def test_sidecar_search_final_bit_exact(dev, rows, dim, nq, k, over):
    """SegmentedIndex::search_final on a Binary sidecar: k x oversample
    Hamming candidates rescored by exact cosine distance, k kept."""
    rng = np.random.default_rng(rows + k + over)
    v = _corpus(rng, rows, dim)
    ids = [f"id{(i * 7919) % rows:06d}" for i in range(rows)]
    sc = _sidecar(dim)
    sc.add_batch(ids, v)
    sc.build()
    q = (v[:nq] + np.float32(0.05) * rng.standard_normal((nq, dim)).astype(np.float32)).astype(np.float32)
    keys, dist = sc.search_final_keys(q, k, over)
    tau = oi.fit_binary_threshold(v, "median")
    wk, wd = oi.search_final(v, q, k, over, tau, "binary", _string_rank(ids))
    assert np.array_equal(keys, wk)
    assert np.array_equal(_bits(dist), _bits(wd))
    sc.close()


def test_sidecar_reference_known_answers(dev):
    """sidecar.rs:1308-1335 and 1337-1424 through the device sidecar: a
    corpus row queried finds itself at Hamming 0; the Binary retrieve ->
    rescore recovers the brute-force top 5 with the perturbed row 9 first."""
    from test_index_oracle import splitmix_vector
    rows12 = np.stack([splitmix_vector(i + 1, 64) for i in range(12)])
    sc = _sidecar(64)
    for i, r in enumerate(rows12):
        sc.add(f"row-{i}", r)
    sc.build()
    assert sc.search(rows12[5], 1) == [("row-5", 0.0)]
    sc.close()
    rows24 = np.stack([splitmix_vector(i + 100, 64) for i in range(24)])
    sc = _sidecar(64)
    sc.add_batch([f"row-{i}" for i in range(24)], rows24)
    sc.build()
    q = (rows24[9] + np.float32(0.05) * splitmix_vector(999, 64)).astype(np.float32)
    got = sc.search_final(q, 5, 32)
    d = np.array([oi.cosine_distance_loop(q, r) for r in rows24], np.float32)
    want = sorted(range(24), key=lambda i: (oi.total_keys(d[i:i + 1])[0], f"row-{i}"))[:5]
    assert [rid for rid, _ in got] == [f"row-{i}" for i in want]
    assert got[0][0] == "row-9"
    sc.close()


def test_sidecar_empty_unbuilt_and_limits(dev):
    from jammi_b200._lib import JbError
    sc = _sidecar(16)
    assert sc.search(np.ones(16, np.float32), 3) == []
    keys, dist = sc.search_keys(np.ones((2, 16), np.float32), 4)
    assert (keys == -1).all() and np.isinf(dist).all()
    sc.add_batch(["x", "y"], np.ones((2, 16), np.float32))
    with pytest.raises(JbError):  # Binary: no threshold until built
        sc.search_keys(np.ones(16, np.float32), 1)
    sc.build()
    keys, _ = sc.search_keys(np.ones(16, np.float32), 4)
    assert keys[0].tolist() == [0, 1, -1, -1]
    with pytest.raises(JbError):  # more candidates than one selection holds
        sc.search_final_keys(np.ones(16, np.float32), 64, 32)
    sc.add("z", np.zeros(16, np.float32))  # an add after the build clears it
    with pytest.raises(JbError):
        sc.search_keys(np.ones(16, np.float32), 1)
    sc.close()


def test_generated_embeddings_into_sidecar(dev, tmp_path):
    """The embedding job's output (values + validity bitmap from
    jb_generate_embeddings) goes straight into the sidecar: the ok rows in
    row order, then build, search_final and the bundle's vector files."""
    from jammi_b200 import Bert
    from jammi_b200.driver import generate_embeddings, pack_rows
    from jammi_b200.synthetic import bert_weights
    cfg = dict(hidden_size=256, num_hidden_layers=2, num_attention_heads=4, intermediate_size=1024,
               vocab_size=4096, max_position_embeddings=128, type_vocab_size=2, layer_norm_eps=1e-12,
               model_type="bert")
    model = Bert.from_weights(bert_weights(cfg, seed=5), cfg, device=0, fmt="bf16")
    rng = np.random.default_rng(6)
    lens = rng.integers(1, 128, size=600)
    lens[[0, 17, 599]] = 0
    rows = [rng.integers(5, 4096, size=n).astype(np.uint32) for n in lens]
    values, offsets = pack_rows(rows)
    out, validity, _ = generate_embeddings([model], values, offsets, batch_rows=128)
    model.close()
    ids = [f"doc-{i:04d}" for i in range(len(rows))]
    sc = _sidecar(256)
    assert sc.write_batch(out, validity, ids) == int((lens > 0).sum())
    n, built = sc.finalize()
    assert n == int((lens > 0).sum()) and built is sc
    store = oi.sidecar_add(out, validity)
    assert np.array_equal(_bits(sc.exact_vectors()), _bits(store))
    assert "doc-0017" not in sc.row_index
    keys, dist = sc.search_final_keys(store[:4], 5, 32)
    kept = [ids[i] for i in range(len(rows)) if lens[i] > 0]
    tau = oi.fit_binary_threshold(store, "median")
    wk, wd = oi.search_final(store, store[:4], 5, 32, tau, "binary", _string_rank(kept))
    assert np.array_equal(keys, wk) and np.array_equal(_bits(dist), _bits(wd))
    assert keys[:, 0].tolist() == [0, 1, 2, 3]  # each stored row finds itself first
    sc.save(str(tmp_path / "emb"))
    assert np.array_equal(np.fromfile(tmp_path / "emb.rawf32", np.float32).reshape(-1, 256), store)
    assert np.array_equal(np.fromfile(tmp_path / "emb.threshold", np.float32), tau)
    raw = (tmp_path / "emb.rowmap").read_bytes()
    assert raw[:4] == (1).to_bytes(4, "little")  # rowmap version, then (u32 length, UTF-8 id) per key
    assert raw[4:8] == (8).to_bytes(4, "little") and raw[8:16] == b"doc-0001" == kept[0].encode()
    sc.close()
