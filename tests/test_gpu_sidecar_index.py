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
