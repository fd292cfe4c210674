"""The CPU oracle pinned against the reference's own known-answer tests.

The reference (MLX + Metal, macOS) cannot run here, so these restate its
test cases; every GPU parity test then compares the CUDA path with this
oracle.
"""

import json
import os

import numpy as np
import pytest

from oracle import oracle as O
from tests import data

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def test_ties_keep_lowest_ids():
    # tests/test_knn.cpp:176-184: ids 1..10 skipping multiples of 97
    x, q = data.ties_rows()
    ids, dist = O.brute_force_knn(x, q, 10, "l2")
    want = [w for w in range(1, 12) if w % 97 != 0][:10]
    assert ids.tolist() == [want, want]
    assert (dist == 0).all()


def test_hamming_tiny_kat():
    # python/tests/test_cuvs.py:844-849
    codes = np.array([[0b1111, 0], [0b1, 0]], dtype=np.uint8)
    ids, dist = O.hamming_knn(codes, codes[:1], 2)
    assert ids[0].tolist() == [0, 1]
    assert dist[0].tolist() == [0.0, 3.0]


def test_fewer_rows_than_k():
    # python/tests/test_mlxvs.py:63-69
    b, q = data.normal_rows(5, 8, 3), data.normal_rows(4, 8, 4)
    ids, dist = O.brute_force_knn(b, q, 8, "l2")
    assert (ids[:, :5] >= 0).all() and (ids[:, 5:] == -1).all()
    assert np.isinf(dist[:, 5:]).all() and (dist[:, 5:] > 0).all()
    assert sorted(ids[0, :5].tolist()) == list(range(5))
    ids, dist = O.brute_force_knn(b, q, 8, "inner_product")
    assert (ids[:, 5:] == -1).all() and np.isneginf(dist[:, 5:]).all()


@pytest.mark.parametrize("metric", ["inner_product", "l2", "cosine"])
@pytest.mark.parametrize("k", [10, 100, 256])
def test_recall_and_distances_vs_float64(metric, k):
    # python/tests/test_mlxvs.py:30-48
    b, q = data.normal_rows(3000, 48, 1), data.normal_rows(32, 48, 2)
    ids, dist = O.brute_force_knn(b, q, k, metric)
    scores = data.exact_scores(metric, q, b)
    assert data.recall(ids, scores, k) == 1.0
    expected = -scores if metric == "l2" else scores
    got = np.take_along_axis(expected, ids, axis=1)
    assert np.allclose(got, dist, rtol=1e-4, atol=1e-4)
    step = np.diff(dist, axis=1)
    assert (step >= -1e-5).all() if metric == "l2" else (step <= 1e-5).all()


def test_integer_data_is_exact():
    # configs 0/1/3: integer-valued rows give exact squared distances
    b, q = data.gaussian_mixture_int(2000, 128, 16, seed=5, nq=20)
    ids, dist = O.brute_force_knn(b, q, 10, "l2")
    exact = ((q.astype(np.int64)[:, None, :] - b.astype(np.int64)[None]) ** 2).sum(-1)
    order = np.lexsort((np.broadcast_to(np.arange(b.shape[0]), exact.shape), exact), axis=1)
    assert (ids == order[:, :10]).all()
    assert (dist == np.take_along_axis(exact, order[:, :10], 1)).all()


def test_hamming_vs_popcount():
    # tests/test_ivf.cpp:252-311 (clustered codes, exact distances), with
    # ids checked too: (distance, id) order
    rows, q = data.hamming_codes(4000, 32, 40, 0.1, seed=7, nq=50)
    ids, dist = O.hamming_knn(rows, q, 10)
    x = np.unpackbits(rows[None, :, :] ^ q[:, None, :], axis=2).sum(2)
    order = np.lexsort((np.broadcast_to(np.arange(rows.shape[0]), x.shape), x), axis=1)
    assert (ids == order[:, :10]).all()
    assert (dist == np.take_along_axis(x, order[:, :10], 1)).all()


def test_merge_keys_is_global_topk():
    b, q = data.gaussian_mixture_int(3000, 32, 8, seed=9, nq=16)
    full = O.knn_keys(b, q, 10, "l2")
    parts = [O.knn_keys(b[i:i + 1000], q, 10, "l2", id_offset=i) for i in range(0, 3000, 1000)]
    merged = O.merge_keys(np.stack(parts), 10)
    assert (merged == full).all()


def test_merge_keys_takes_repeated_keys_once():
    # lists sharing keys (the GPU search's units start from an earlier
    # unit's list), in any order, with empty slots
    rng = np.random.default_rng(5)
    L, nq, k = 9, 40, 10
    ids = rng.integers(0, 60, size=(L, nq, k))
    table = rng.integers(-20, 20, size=(nq, 60)).astype(np.float32)
    scores = np.take_along_axis(table[None].repeat(L, 0), ids, axis=2)
    keys = np.vectorize(lambda s, i: O.key(float(s), int(i)), otypes=[np.uint64])(scores, ids)
    keys[rng.random(keys.shape) < 0.2] = 0
    merged = O.merge_keys(keys, k)
    for i in range(nq):
        u = np.unique(keys[:, i, :])[::-1]
        u = u[u != 0][:k]
        assert (merged[i, :len(u)] == u).all() and (merged[i, len(u):] == 0).all()


def test_key_order():
    # higher score first, then lower id (src/kernels.h:20-23)
    assert O.key(2.0, 5) > O.key(1.0, 0)
    assert O.key(1.0, 3) > O.key(1.0, 4)
    assert O.key(-1.0, 0) > O.key(-2.0, 0)
    assert O.key(float("-inf"), 7) > 0
    ids, scores = O.decode_keys(np.array([O.key(1.5, 12), 0], np.uint64))
    assert ids.tolist() == [12, -1] and scores[0] == 1.5 and np.isneginf(scores[1])


def test_golden_fixtures():
    """Committed fixtures (tests/golden/make_golden.py) reproduce exactly."""
    with open(os.path.join(GOLDEN, "golden.json")) as f:
        cases = json.load(f)
    for case in cases:
        hamming, b, q = data.golden_inputs(case["input"])
        if hamming:
            ids, dist = O.hamming_knn(b, q, case["k"])
        else:
            ids, dist = O.brute_force_knn(b, q, case["k"], case["metric"])
        assert ids.tolist() == case["ids"], case["name"]
        if case.get("exact", True):
            assert dist.tolist() == case["distances"], case["name"]
        else:
            assert np.allclose(dist, np.array(case["distances"], np.float32), rtol=1e-5,
                               atol=1e-5), case["name"]


def test_invalid_arguments():
    b = data.normal_rows(10, 4, 1)
    with pytest.raises(ValueError):
        O.brute_force_knn(b, b, 300, "l2")
    with pytest.raises(ValueError):
        O.brute_force_knn(b, b, 0, "l2")


def test_all_neighbors_small_n_kats():
    # python/tests/test_mlxvs.py:192-195: 5 rows, k = 8: the 4 other rows,
    # then -1; tests/test_all_neighbors.cpp:76-98: 10 rows, k = 32: every
    # other row once, then -1
    ids, dist = O.all_neighbors(data.normal_rows(5, 4, 1), 8, "l2")
    assert (ids[:, :4] >= 0).all() and (ids[:, 4:] == -1).all()
    assert np.isinf(dist[:, 4:]).all()
    ids, _ = O.all_neighbors(data.normal_rows(10, 7, 21), 32, "l2")
    for i in range(10):
        assert sorted(ids[i, :9].tolist()) == [j for j in range(10) if j != i]
        assert (ids[i, 9:] == -1).all()


@pytest.mark.parametrize("metric", ["l2", "inner_product"])
def test_all_neighbors_is_self_excluded_topk(metric):
    # the k + 1 search and merge_lists equal the top k of every other row
    # (integer data: exact scores, ties to the lower id)
    x, _ = data.gaussian_mixture_int(600, 16, 6, seed=5)
    x = np.rint(x / 16.0).astype(np.float32)  # many ties
    k = 12
    ids, dist = O.all_neighbors(x, k, metric)
    scores = data.exact_scores(metric, x, x)
    np.fill_diagonal(scores, -np.inf)
    order = np.lexsort((np.broadcast_to(np.arange(600), scores.shape), -scores), axis=1)[:, :k]
    assert np.array_equal(ids, order)
    want = np.take_along_axis(scores, order, 1)
    assert np.array_equal(dist, (-want if metric == "l2" else want).astype(np.float32))


def test_topk_merge_oracle_order():
    # the running list and the new scores merged: best score first, equal
    # scores by id as unsigned (-1 last), src/kernels.h:21-23
    rng = np.random.default_rng(7)
    s = rng.integers(0, 4, (5, 40)).astype(np.float32)
    ids0, sc0 = O.topk_merge(s, None, None, 50, True, 12)
    ids1, sc1 = O.topk_merge(s, ids0, sc0, 7, False, 12)
    for i in range(5):
        cand = [(float(v), 50 + j) for j, v in enumerate(s[i])] + \
               [(float(v), 7 + j) for j, v in enumerate(s[i])]
        cand.sort(key=lambda e: (-e[0], e[1] & 0xFFFFFFFF))
        assert ids1[i].tolist() == [e[1] for e in cand[:12]]
        assert sc1[i].tolist() == [e[0] for e in cand[:12]]
    # fewer entries than k: -1 / -inf padding
    ids, sc = O.topk_merge(s[:, :3], None, None, 0, True, 5)
    assert (ids[:, 3:] == -1).all() and np.isneginf(sc[:, 3:]).all()


def test_refine_oracle_matches_exact():
    x, _ = data.gaussian_mixture_int(300, 16, 4, seed=9)
    q = x[:20]
    rng = np.random.default_rng(3)
    cand = rng.integers(-5, 320, (20, 30))
    ids, dist = O.refine(x, q, cand, 8, "l2")
    for i in range(20):
        rows = [(int(((x[c] - q[i]) ** 2).sum()), j, c) for j, c in enumerate(cand[i])
                if 0 <= c < 300]
        rows.sort(key=lambda e: (e[0], e[1]))
        want = [c for _, _, c in rows[:8]] + [-1] * max(0, 8 - len(rows))
        assert ids[i].tolist() == want
