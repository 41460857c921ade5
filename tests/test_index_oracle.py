"""Pin the index oracle (oracle/index.py) to the reference's own known answers
for the sidecar's threshold packing, exact search and cosine distance, and
to scalar restatements.  CPU only."""
import numpy as np

from oracle import index as oi


# crates/jammi-db/src/index/sidecar.rs:1280-1294
def test_pack_zero_threshold_known_answer():
    v = np.array([1.0, -1.0, 0.0, 2.0, -0.5, 0.5, -3.0, 4.0, 0.1], np.float32)
    packed = oi.pack_threshold_bits(v, np.zeros(9, np.float32))[0]
    assert list(packed) == [0b1010_1001, 0b0000_0001]


# sidecar.rs:1296-1306
def test_pack_per_dimension_threshold_known_answer():
    packed = oi.pack_threshold_bits(np.array([0.4, 0.6, -0.1, -0.1], np.float32),
                                    np.array([0.5, 0.5, -0.2, 0.0], np.float32))[0]
    assert list(packed) == [0b0000_0110]


# crates/jammi-db/tests/it/index.rs:169-245: "near" first, every row scored
def test_exact_search_known_answer():
    corpus = np.array([[0, 1, 0, 0], [1, 0, 0, 0], [0.7, 0.7, 0, 0], [-1, 0, 0, 0]], np.float32)
    idx, dist = oi.exact_search(corpus, np.array([[1, 0, 0, 0]], np.float32), 4)
    assert list(idx[0]) == [1, 2, 0, 3]  # near, mid, far, opp
    assert dist[0, 0] == 0.0 and dist[0, 2] == 1.0 and dist[0, 3] == 2.0


def test_cosine_distance_conventions():
    # a zero-magnitude side gives distance 1 (distance.rs:16-19)
    assert oi.cosine_distance_loop([0, 0, 0], [1, 2, 3]) == np.float32(1.0)
    assert oi.cosine_distances(np.zeros(3, np.float32), np.eye(3, dtype=np.float32)).tolist() == [1, 1, 1]


def test_vectorised_distance_equals_scalar_loop():
    rng = np.random.default_rng(0)
    c = rng.standard_normal((40, 37)).astype(np.float32)
    q = rng.standard_normal(37).astype(np.float32)
    c[3] = 0
    got = oi.cosine_distances(q, c)
    want = np.array([oi.cosine_distance_loop(q, row) for row in c], np.float32)
    assert got.view(np.uint32).tolist() == want.view(np.uint32).tolist()


def test_exact_search_ties_follow_rank():
    corpus = np.tile(np.array([[1.0, 2.0, 3.0]], np.float32), (5, 1))
    rank = np.array([4, 2, 0, 3, 1])
    idx, _ = oi.exact_search(corpus, corpus[:1], 5, tie_rank=rank)
    assert list(idx[0]) == [2, 4, 1, 3, 0]
    idx, _ = oi.exact_search(corpus, corpus[:1], 3)
    assert list(idx[0]) == [0, 1, 2]


def test_mean_threshold_is_the_row_order_f64_sum():
    rng = np.random.default_rng(1)
    v = (rng.standard_normal((257, 3)) * 1e3).astype(np.float32)
    want = []
    for d in range(3):
        s = 0.0
        for r in range(257):
            s += float(v[r, d])
        want.append(np.float32(s / 257))
    assert oi.fit_binary_threshold(v, "mean").tolist() == want


def test_median_threshold_even_odd_and_total_order():
    v = np.array([[3.0], [1.0], [2.0]], np.float32)
    assert oi.fit_binary_threshold(v, "median")[0] == 2.0
    v = np.array([[4.0], [1.0], [3.0], [2.0]], np.float32)
    assert oi.fit_binary_threshold(v, "median")[0] == 2.5
    # total order puts -0.0 before +0.0; their average is +0.0
    v = np.array([[0.0], [-0.0]], np.float32)
    assert oi.fit_binary_threshold(v, "median").view(np.uint32)[0] == 0
    # a NaN sorts after every number
    v = np.array([[np.nan], [5.0], [1.0]], np.float32)
    assert oi.fit_binary_threshold(v, "median")[0] == 5.0
    assert oi.fit_binary_threshold(np.zeros((0, 4), np.float32), "median").tolist() == [0, 0, 0, 0]


def test_threshold_reads_only_the_first_100000_rows():
    v = np.zeros((oi.SAMPLE_CAP + 3, 2), np.float32)
    v[: oi.SAMPLE_CAP] = 1.0
    v[oi.SAMPLE_CAP:] = 1e30
    assert oi.fit_binary_threshold(v, "mean").tolist() == [1.0, 1.0]
    assert oi.fit_binary_threshold(v, "median").tolist() == [1.0, 1.0]


# The reference's sidecar tests draw their corpora from splitmix64
# (sidecar.rs:1261-1278): value = (bits >> 11) / 2^53 * 2 - 1 as f32.
def splitmix_vector(seed: int, dim: int) -> np.ndarray:
    mask = (1 << 64) - 1
    state, out = seed, []
    for _ in range(dim):
        state = (state + 0x9E3779B97F4A7C15) & mask
        z = state
        z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & mask
        z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & mask
        z ^= z >> 31
        out.append(np.float32((z >> 11) / float(1 << 53) * 2.0 - 1.0))
    return np.array(out, np.float32)


def string_rank(ids):
    order = sorted(range(len(ids)), key=ids.__getitem__)
    rank = np.empty(len(ids), np.int64)
    rank[order] = np.arange(len(ids))
    return rank


# sidecar.rs:1308-1335: a query equal to corpus row 5 is its own nearest, at
# Hamming distance 0 (median tau, the reference's build default)
def test_binary_query_is_its_own_nearest_at_hamming_zero():
    store = np.stack([splitmix_vector(i + 1, 64) for i in range(12)])
    tau = oi.fit_binary_threshold(store, "median")
    ids = [f"row-{i}" for i in range(12)]
    keys, dist = oi.sidecar_search(store, store[5:6], 1, "binary", tau, string_rank(ids))
    assert keys[0, 0] == 5 and dist[0, 0] == 0.0


# sidecar.rs:1337-1424: retrieve -> rescore with the Binary oversample (32)
# over 24 rows recovers the exact brute-force top 5, the perturbed row 9 first
def test_binary_retrieve_rescore_matches_exact_top_k():
    store = np.stack([splitmix_vector(i + 100, 64) for i in range(24)])
    ids = [f"row-{i}" for i in range(24)]
    rank = string_rank(ids)
    q = (store[9] + np.float32(0.05) * splitmix_vector(999, 64)).astype(np.float32)
    tau = oi.fit_binary_threshold(store, "median")
    keys, dist = oi.search_final(store, q[None, :], 5, 32, tau, "binary", rank)
    d = np.array([oi.cosine_distance_loop(q, row) for row in store], np.float32)
    expected = sorted(range(24), key=lambda i: (oi.total_keys(d[i:i + 1])[0], ids[i]))[:5]
    assert keys[0].tolist() == expected
    assert keys[0, 0] == 9
    assert dist[0].view(np.uint32).tolist() == d[expected].view(np.uint32).tolist()


def test_sidecar_add_keeps_valid_rows_in_order():
    v = np.arange(10 * 3, dtype=np.float32).reshape(10, 3)
    bits = np.packbits(np.array([1, 0, 0, 1, 1, 0, 1, 0, 0, 1], bool), bitorder="little")
    assert oi.sidecar_add(v, bits)[:, 0].tolist() == [0, 9, 12, 18, 27]
    assert oi.sidecar_add(v, None).shape == (10, 3)


def test_search_final_on_exact_store_is_search():
    rng = np.random.default_rng(3)
    store = rng.standard_normal((30, 16)).astype(np.float32)
    q = rng.standard_normal((2, 16)).astype(np.float32)
    a = oi.search_final(store, q, 4, 32, None, "f32")
    b = oi.exact_search(store, q, 4)
    assert np.array_equal(a[0], b[0]) and np.array_equal(a[1], b[1])


def test_sidecar_search_pads_past_the_store():
    store = np.eye(3, dtype=np.float32)
    keys, dist = oi.sidecar_search(store, store[:1], 5, "f32")
    assert keys[0].tolist()[:3] == [0, 1, 2] and keys[0].tolist()[3:] == [-1, -1]
    assert np.isinf(dist[0, 3:]).all()
