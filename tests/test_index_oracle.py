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
