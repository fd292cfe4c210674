"""GPU parity of all_neighbors (exact, one cluster) against the CPU oracle,
which restates the reference's k + 1 search and merge_lists
(src/all_neighbors.cpp:56-95,250-263).  The library excludes each row's own
id inside the fused kernel instead.

Contract as brute_force_knn: integer data bit-exact (ids and distances),
float data tie-tolerant recall 1.0 with distances within 1e-4, the row
itself never listed, -1 / +-inf padding when fewer than k other rows exist.
"""

import numpy as np
import pytest

import mlxvs_b200 as mv
from oracle import oracle as O
from tests import data

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("metric,k", [("l2", 32), ("inner_product", 10), ("l2", 100)])
def test_integer_rows_bit_exact(metric, k):
    # config 3 shape at small n: the config-1 mixture, k = 32
    x, _ = data.gaussian_mixture_int(20_000, 128, 64, seed=51)
    ids, dist = mv.all_neighbors(x, k, metric, algo="brute_force")
    oids, odist = O.all_neighbors(x, k, metric)
    assert np.array_equal(ids, oids)
    assert np.array_equal(dist, odist)
    assert not (ids == np.arange(x.shape[0])[:, None]).any()


def test_duplicates_and_ties():
    # repeated rows: the twin (distance 0) is a neighbor, the row itself is
    # not; coarse integers give many equal distances (lower id first)
    x, _ = data.gaussian_mixture_int(3_000, 16, 8, seed=52)
    x = np.rint(x / 20.0).astype(np.float32)
    x = np.concatenate([x, x[:500]])
    ids, dist = mv.all_neighbors(x, 16, "l2", algo="brute_force")
    oids, odist = O.all_neighbors(x, 16, "l2")
    assert np.array_equal(ids, oids)
    assert np.array_equal(dist, odist)
    assert (ids[:500, 0] >= 3_000).all() and (dist[:500, 0] == 0).all()


@pytest.mark.parametrize("metric", ["l2", "cosine", "inner_product"])
def test_float_rows_recall_and_tolerance(metric):
    x = data.normal_rows(6_000, 48, seed=53)
    k = 12
    ids, dist = mv.all_neighbors(x, k, metric, algo="brute_force")
    scores = data.exact_scores(metric, x, x)
    np.fill_diagonal(scores, -np.inf)
    assert data.recall(ids, scores, k, tol=1e-4) == 1.0
    want = np.take_along_axis(scores, ids.astype(np.int64), 1)
    want = -want if metric == "l2" else want
    assert np.allclose(dist, want, rtol=1e-4, atol=1e-4)
    assert not (ids == np.arange(x.shape[0])[:, None]).any()


def test_small_n_kats():
    # python/tests/test_mlxvs.py:192-195 (default algo: n <= brute_force_below
    # takes the exact build) and tests/test_all_neighbors.cpp:76-98
    ids, dist = mv.all_neighbors(data.normal_rows(5, 4, 1), 8, "l2")
    assert (ids[:, :4] >= 0).all() and (ids[:, 4:] == -1).all()
    assert np.isinf(dist[:, 4:]).all()
    ids, _ = mv.all_neighbors(data.normal_rows(10, 7, 21), 32, "l2")
    for i in range(10):
        assert sorted(ids[i, :9].tolist()) == [j for j in range(10) if j != i]
        assert (ids[i, 9:] == -1).all()


def test_bad_input():
    # python/tests/test_mlxvs.py:196-201
    z = np.zeros((10, 4), np.float32)
    with pytest.raises(ValueError):
        mv.all_neighbors(z, 200)
    with pytest.raises(ValueError):
        mv.all_neighbors(z, 4, n_clusters=11)
    with pytest.raises(ValueError):
        mv.all_neighbors(z, 4, n_clusters=2, overlap_factor=3)
    with pytest.raises(ValueError):
        mv.all_neighbors(z[:1], 4, algo="brute_force")
    with pytest.raises(NotImplementedError):
        mv.all_neighbors(np.zeros((5000, 4), np.float32), 4)  # NN-Descent build
    with pytest.raises(NotImplementedError):
        mv.all_neighbors(z, 4, algo="brute_force", n_clusters=2)


def test_device_tensors_and_row_ranges():
    import torch

    x, _ = data.gaussian_mixture_int(9_000, 64, 16, seed=54)
    hids, hdist = mv.all_neighbors(x, 20, "l2", algo="brute_force")
    tx = torch.from_numpy(x).cuda()
    ids, dist = mv.all_neighbors(tx, 20, "l2", algo="brute_force")
    torch.cuda.synchronize()
    assert ids.is_cuda and np.array_equal(ids.cpu().numpy(), hids)
    assert np.array_equal(dist.cpu().numpy(), hdist)
    # the rows of one device when devices split the graph by rows
    for b, e in [(0, 4_000), (4_000, 9_000), (1_234, 1_235), (7, 7)]:
        rids, rdist = mv.all_neighbors_rows(tx, 20, "l2", begin=b, end=e)
        torch.cuda.synchronize()
        assert np.array_equal(rids.cpu().numpy(), hids[b:e])
        assert np.array_equal(rdist.cpu().numpy(), hdist[b:e])
    mv.synchronize()
