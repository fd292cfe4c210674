"""The cuVS-style front end ``mlxvs_b200.cuvs.neighbors.brute_force``
(python/mlxvs/cuvs/neighbors/brute_force.py; its tests
python/tests/test_cuvs.py:147-221,777-793).

CPU: the metric table, the distance conversion and the refusals.
GPU: searches through the sm_100a kernels, bit-exact against the oracle on
integer data for the L2 and inner-product metrics and on Hamming codes,
recall 1 for cosine, host and CUDA inputs, outputs written in place."""

import numpy as np
import pytest

from mlxvs_b200.cuvs import distance as D
from mlxvs_b200.cuvs.neighbors import brute_force as bf
from oracle import oracle as O
from tests import data

FAST_METRICS = ["sqeuclidean", "euclidean", "l2", "inner_product", "cosine"]


def test_metric_table():
    # python/mlxvs/cuvs/distance.py:11-56
    assert D.metric_type("sqeuclidean") == D.L2Expanded == 0
    assert D.metric_type("l2") == D.metric_type("euclidean") == D.L2SqrtExpanded == 1
    assert D.metric_type("cosine") == 2 and D.metric_type("inner_product") == 6
    assert D.metric_type("bitwise_hamming") == 20 and D.metric_type(6) == 6
    with pytest.raises(ValueError):
        D.metric_type("nope")
    assert repr(bf.build(np.zeros((2, 2), np.float32), "cosine")) == \
        "Index(type=BruteForce, metric=cosine)"


def test_to_cuvs_distances():
    # python/mlxvs/cuvs/neighbors/_common.py:39-48
    s = np.array([[-1.0, 0.0, 4.0, np.inf]], np.float32)
    assert np.array_equal(D.to_cuvs_distances(s, D.L2Expanded), [[0, 0, 4, np.inf]])
    assert np.array_equal(D.to_cuvs_distances(s, D.L2SqrtExpanded), [[0, 0, 2, np.inf]])
    c = np.array([[1.0, 0.5, -np.inf]], np.float32)
    assert np.array_equal(D.to_cuvs_distances(c, D.CosineExpanded), [[0, 0.5, np.inf]])
    assert D.to_cuvs_distances(c, D.InnerProduct) is c


def test_refusals_before_any_search():
    x = np.zeros((4, 2), np.float32)
    with pytest.raises(ValueError, match="built"):
        bf.search(bf.Index(), x, 1)
    with pytest.raises(NotImplementedError, match="cityblock"):
        bf.search(bf.build(x, "cityblock"), x, 1)

    class Bitset:
        type = "bitset"

    with pytest.raises(NotImplementedError, match="prefilter"):
        bf.search(bf.build(x), x, 1, prefilter=Bitset())
    with pytest.raises(ValueError, match="matrix"):
        bf.build(np.zeros(3, np.float32))


# --- searches on the GPU -------------------------------------------------------


def _oracle_cuvs(b, q, k, metric):
    """The oracle's ids and scores as cuVS's int64 ids and float32 distances."""
    t = D.metric_type(metric)
    ids, scores = O.brute_force_knn(b, q, k, D.FAST[t])
    return ids.astype(np.int64), D.to_cuvs_distances(scores, t)


@pytest.mark.gpu
@pytest.mark.parametrize("metric", ["sqeuclidean", "euclidean", "inner_product"])
@pytest.mark.parametrize("where", ["host", "cuda"])
def test_integer_rows_bit_exact(metric, where):
    import torch

    b, q = data.gaussian_mixture_int(20_000, 128, 32, seed=51, nq=300)
    oids, odist = _oracle_cuvs(b, q, 10, metric)
    if where == "cuda":
        idx = bf.build(torch.from_numpy(b).cuda(), metric)
        d, i = bf.search(idx, torch.from_numpy(q).cuda(), 10)
        assert d.is_cuda and i.is_cuda
        d, i = d.cpu().numpy(), i.cpu().numpy()
    else:
        d, i = bf.search(bf.build(b, metric), q, 10)
    assert i.dtype == np.int64 and d.dtype == np.float32
    assert np.array_equal(i, oids)
    assert np.array_equal(d, odist)


@pytest.mark.gpu
@pytest.mark.parametrize("metric", FAST_METRICS)
@pytest.mark.parametrize("inplace", [True, False])
def test_uniform_rows_as_reference(metric, inplace):
    # python/tests/test_cuvs.py:162-194 for the metrics the GPU search runs
    rng = np.random.default_rng(3)
    index = rng.random((100, 40)).astype(np.float32)
    queries = rng.random((32, 40)).astype(np.float32)
    k = 5
    indices = np.zeros((32, k), np.int64)
    distances = np.zeros((32, k), np.float32)
    idx = bf.build(index, metric)
    ret_d, ret_i = bf.search(idx, queries, k, neighbors=indices if inplace else None,
                             distances=distances if inplace else None)
    got = (distances if inplace else ret_d).copy()
    ids = indices if inplace else ret_i
    assert ids.dtype == np.int64
    q64, b64 = queries.astype(np.float64), index.astype(np.float64)
    if metric == "inner_product":
        pw = -(q64 @ b64.T)
        want = -np.sort(pw, axis=1)[:, :k]
    else:
        sq = ((q64[:, None] - b64[None]) ** 2).sum(-1)
        if metric == "sqeuclidean":
            pw = sq
        elif metric == "cosine":
            qn = q64 / np.linalg.norm(q64, axis=1, keepdims=True)
            bn = b64 / np.linalg.norm(b64, axis=1, keepdims=True)
            pw = 1 - qn @ bn.T
        else:
            pw = np.sqrt(sq)
        want = np.sort(pw, axis=1)[:, :k]
    got[np.abs(got) <= 1e-5] = 0.0
    np.testing.assert_allclose(got, want, atol=1e-3, rtol=1e-3)
    # the returned ids are rows at the returned distances
    at = np.take_along_axis(pw, ids, 1)
    np.testing.assert_allclose(np.abs(at), np.abs(want), atol=1e-3, rtol=1e-3)


@pytest.mark.gpu
def test_cosine_recall_and_cuda_inplace():
    import torch

    b, q = data.lowrank_unit(30_000, 96, 16, seed=52, nq=200)
    dev = torch.device("cuda", 0)
    nb = torch.zeros((200, 10), dtype=torch.int64, device=dev)
    dd = torch.zeros((200, 10), dtype=torch.float32, device=dev)
    d, i = bf.search(bf.build(torch.from_numpy(b).to(dev), "cosine"), q, 10,
                     neighbors=nb, distances=dd)
    assert d is dd and i is nb
    scores = data.exact_scores("cosine", q, b)
    assert data.recall(i.cpu().numpy(), scores, 10, tol=1e-4) == 1.0
    want = 1 - np.take_along_axis(scores, i.cpu().numpy(), 1)
    np.testing.assert_allclose(d.cpu().numpy(), want, atol=1e-4, rtol=1e-4)


@pytest.mark.gpu
@pytest.mark.parametrize("metric,pad", [("sqeuclidean", np.inf), ("euclidean", np.inf),
                                        ("cosine", np.inf), ("inner_product", -np.inf),
                                        ("bitwise_hamming", np.inf)])
def test_more_neighbors_than_rows(metric, pad):
    rng = np.random.default_rng(7)
    if metric == "bitwise_hamming":
        x = rng.integers(0, 256, (3, 8), dtype=np.uint8)
    else:
        x = rng.random((3, 8)).astype(np.float32)
    d, i = bf.search(bf.build(x, metric), x, 5)
    assert (i[:, :3] >= 0).all() and (i[:, 3:] == -1).all()
    assert (d[:, 3:] == pad).all()


def _hamming(a, b):
    return np.unpackbits(a[:, None] ^ b[None], axis=2).sum(2)


@pytest.mark.gpu
@pytest.mark.parametrize("bytes_", [3, 16, 128])
def test_bitwise_hamming_as_reference(bytes_):
    # python/tests/test_cuvs.py:777-793 without the prefilter, and bit-exact
    # against the oracle (ties to the lower id)
    rng = np.random.default_rng(11)
    codes = rng.integers(0, 256, (700, bytes_), dtype=np.uint8)
    queries = rng.integers(0, 256, (40, bytes_), dtype=np.uint8)
    index = bf.build(codes, metric="bitwise_hamming")
    d, i = bf.search(index, queries, 7)
    want = np.sort(_hamming(queries, codes), axis=1)[:, :7]
    np.testing.assert_array_equal(d, want)
    np.testing.assert_array_equal(np.take_along_axis(_hamming(queries, codes), i, 1), want)
    oids, odist = O.hamming_knn(codes, queries, 7)
    assert np.array_equal(i, oids.astype(np.int64)) and np.array_equal(d, odist)


@pytest.mark.gpu
def test_bitwise_hamming_cuda_codes():
    import torch

    rows, q = data.hamming_codes(50_000, 128, 512, 0.1, seed=53, nq=120)
    d, i = bf.search(bf.build(torch.from_numpy(rows).cuda(), "bitwise_hamming"), q, 10)
    oids, odist = O.hamming_knn(rows, q, 10)
    assert i.dtype == torch.int64 and d.dtype == torch.float32
    assert np.array_equal(i.cpu().numpy(), oids) and np.array_equal(d.cpu().numpy(), odist)
