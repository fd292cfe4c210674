"""GPU parity of brute_force_knn (the C API, sm_100a kernels) against the CPU
oracle and the reference's known-answer tests.

Contract (restated per case):
  - integer-valued inputs (configs 0/1/3): ids and distances bit-exact
    (every product and partial sum is an integer below 2^24, so the
    reference's float32 results are exact);
  - general float32 inputs: tie-tolerant recall@k == 1.0 and distances
    within rtol = atol = 1e-4 of float64 (python/tests/test_mlxvs.py:45);
  - ties keep the lowest ids, identically on every run.
"""

import json
import os

import numpy as np
import pytest

import mlxvs_b200 as mv
from oracle import oracle as O
from tests import data

pytestmark = pytest.mark.gpu

RTOL = ATOL = 1e-4


def check_float(metric, b, q, k, ids, dist):
    scores = data.exact_scores(metric, q, b)
    keff = min(k, b.shape[0])
    assert data.recall(ids[:, :keff], scores, keff, tol=1e-4) == 1.0
    expected = -scores if metric == "l2" else scores
    got = np.take_along_axis(expected, np.maximum(ids[:, :keff], 0), axis=1)
    assert np.allclose(got, dist[:, :keff], rtol=RTOL, atol=ATOL)
    step = np.diff(dist[:, :keff], axis=1)
    assert (step >= -1e-5).all() if metric == "l2" else (step <= 1e-5).all()


def test_config0_bit_exact():
    # 100k x 128 integer mixture, 1k queries, L2, k=10
    b, q = data.gaussian_mixture_int(100_000, 128, 64, seed=0, nq=1000)
    ids, dist = mv.brute_force_knn(b, q, 10, "l2")
    oids, odist = O.brute_force_knn(b, q, 10, "l2")
    assert np.array_equal(ids, oids)
    assert np.array_equal(dist, odist)


@pytest.mark.parametrize("metric", ["l2", "inner_product"])
@pytest.mark.parametrize("k", [1, 10, 33, 100, 256])
def test_integer_data_bit_exact(metric, k):
    b, q = data.gaussian_mixture_int(20_000, 128, 32, seed=3, nq=300)
    ids, dist = mv.brute_force_knn(b, q, k, metric)
    oids, odist = O.brute_force_knn(b, q, k, metric)
    assert np.array_equal(ids, oids)
    assert np.array_equal(dist, odist)


@pytest.mark.parametrize("metric", ["l2", "inner_product"])
@pytest.mark.parametrize("k", [1, 10, 16])
def test_exact_fp16_values_with_fractional_norms(metric, k):
    # quarter steps in [0, 64): every value is exactly an fp16 and every
    # float32 product and sum is exact, but |b|^2 is not an integer, so for
    # L2 it cannot ride in the MMA and the search that was launched before
    # the prep's flags were read must step aside (inner product keeps it)
    b, q = data.gaussian_mixture_int(30_000, 128, 32, seed=11, nq=300)
    b = (b * 0.25).astype(np.float32)
    q = (q * 0.25).astype(np.float32)
    for _ in range(2):
        ids, dist = mv.brute_force_knn(b, q, k, metric)
        oids, odist = O.brute_force_knn(b, q, k, metric)
        assert np.array_equal(ids, oids)
        assert np.array_equal(dist, odist)


@pytest.mark.parametrize("d", [8, 48, 100, 130, 200, 300])
def test_integer_data_odd_dims(d):
    b, q = data.gaussian_mixture_int(5_000 + 17, d, 8, seed=d, nq=77)
    ids, dist = mv.brute_force_knn(b, q, 16, "l2")
    oids, odist = O.brute_force_knn(b, q, 16, "l2")
    assert np.array_equal(ids, oids)
    assert np.array_equal(dist, odist)


def test_ties_keep_lowest_ids_deterministic():
    # tests/test_knn.cpp:158-192
    x, q = data.ties_rows()
    first, _ = mv.brute_force_knn(x, q, 10, "l2")
    want = [w for w in range(1, 12) if w % 97 != 0][:10]
    assert first.tolist() == [want, want]
    for _ in range(20):
        again, _ = mv.brute_force_knn(x, q, 10, "l2")
        assert np.array_equal(again, first)


@pytest.mark.parametrize("metric", ["inner_product", "l2", "cosine"])
@pytest.mark.parametrize("k", [10, 100, 256])
def test_normal_rows_recall_and_tolerance(metric, k):
    # python/tests/test_mlxvs.py:30-48 (general float32: split-fp16 path)
    b, q = data.normal_rows(3000, 48, 1), data.normal_rows(32, 48, 2)
    ids, dist = mv.brute_force_knn(b, q, k, metric)
    assert ids.shape == (32, k) and dist.shape == (32, k)
    check_float(metric, b, q, k, ids, dist)


@pytest.mark.parametrize("metric", ["inner_product", "l2", "cosine"])
def test_reference_sweep(metric):
    # tests/test_knn.cpp:197-207 shapes
    for n, nq, d, k in [(5000, 64, 64, 10), (5000, 64, 96, 96), (5000, 64, 128, 32),
                        (3000, 16, 32, 256), (4000, 32, 64, 1), (5000, 61, 64, 16),
                        (3000, 29, 32, 10)]:
        b, q = data.normal_rows(n, d, 1), data.normal_rows(nq, d, 2)
        ids, dist = mv.brute_force_knn(b, q, k, metric)
        check_float(metric, b, q, k, ids, dist)


def test_unit_rows_config2_shape():
    # config 2 distribution (unit rows with a shared low-rank part), small
    b, q = data.lowrank_unit(20_000, 1536, 64, seed=2, nq=64)
    for metric in ["cosine", "inner_product"]:
        ids, dist = mv.brute_force_knn(b, q, 10, metric)
        check_float(metric, b, q, 10, ids, dist)


def test_float16_storage():
    # float16 inputs are upcast (src/utils.h:28): exact fp16 operands, float32
    # accumulation; compared with float64 of the same fp16 values
    b, q = data.lowrank_unit(20_000, 256, 64, seed=4, nq=64)
    b16 = b.astype(np.float16).astype(np.float32)
    q16 = q.astype(np.float16).astype(np.float32)
    for metric in ["inner_product", "l2"]:
        ids, dist = mv.brute_force_knn(b16, q16, 10, metric)
        check_float(metric, b16, q16, 10, ids, dist)


def test_fewer_rows_than_k():
    # python/tests/test_mlxvs.py:63-69
    b, q = data.normal_rows(5, 8, 3), data.normal_rows(4, 8, 4)
    ids, dist = mv.brute_force_knn(b, q, 8, "l2")
    assert (ids[:, :5] >= 0).all() and (ids[:, 5:] == -1).all()
    assert np.isinf(dist[:, 5:]).all() and (dist[:, 5:] > 0).all()
    assert sorted(ids[0, :5].tolist()) == list(range(5))
    ids, dist = mv.brute_force_knn(b, q, 8, "cosine")
    assert (ids[:, 5:] == -1).all() and np.isneginf(dist[:, 5:]).all()


def test_tiny_shapes():
    # python/tests/test_mlxvs.py:51-60
    b, q = data.normal_rows(100, 8, 21), data.normal_rows(2, 8, 22)
    ids, dist = mv.brute_force_knn(b, q, 3, "cosine")
    check_float("cosine", b, q, 3, ids, dist)
    ids, _ = mv.brute_force_knn(b, q, 1, "l2", tile_rows=7)
    assert ids.shape == (2, 1)
    ids, dist = mv.brute_force_knn(b[:1], q, 4, "l2")
    assert ids[:, 0].tolist() == [0, 0] and (ids[:, 1:] == -1).all()


def test_empty_inputs():
    b = data.normal_rows(10, 4, 1)
    ids, dist = mv.brute_force_knn(b, b[:0], 3, "l2")
    assert ids.shape == (0, 3)
    ids, dist = mv.brute_force_knn(b[:0], b, 3, "l2")
    assert (ids == -1).all() and np.isposinf(dist).all()
    ids, dist = mv.brute_force_knn(b[:0], b, 3, "inner_product")
    assert (ids == -1).all() and np.isneginf(dist).all()


def test_errors():
    # python/tests/test_mlxvs.py:72-78, :240-246
    with pytest.raises(ValueError):
        mv.brute_force_knn(np.zeros((4, 3)), np.zeros((2, 5)), 1)
    with pytest.raises(ValueError):
        mv.brute_force_knn(np.zeros((4, 3)), np.zeros((2, 3)), 300)
    with pytest.raises(ValueError):
        mv.brute_force_knn(np.zeros((4, 3), bool), np.zeros((2, 3)), 1)
    with pytest.raises(ValueError, match="same number of columns"):
        mv.brute_force_knn(data.normal_rows(10, 4, 1), data.normal_rows(10, 5, 1), 2)


def test_non_contiguous_and_dtypes():
    # python/tests/test_mlxvs.py:81-87, :206-225
    b = data.normal_rows(500, 64, 5)
    q = data.normal_rows(8, 64, 6)
    ids_view, _ = mv.brute_force_knn(np.ascontiguousarray(b.T).T, q, 10, "l2")
    ids, _ = mv.brute_force_knn(b, q, 10, "l2")
    assert np.array_equal(ids_view, ids)
    x = data.normal_rows(500, 16, 15)
    want, _ = mv.brute_force_knn(x, x, 5, "l2")
    for conv in (lambda a: a.astype(np.float64), lambda a: a.tolist(),
                 lambda a: a.astype(np.float16)):
        got, _ = mv.brute_force_knn(conv(x), conv(x), 5, "l2")
        assert (got[:, 0] == np.arange(500)).all()
        assert (got == want).mean() > 0.9


def test_metric_names():
    x = data.normal_rows(300, 8, 16)
    for name in ["l2", "cosine", "inner_product"]:
        a, _ = mv.brute_force_knn(x, x, 3, name)
        b, _ = mv.brute_force_knn(x, x, 3, getattr(mv.Metric, name))
        assert (a == b).all()
    with pytest.raises(ValueError, match="unknown Metric 'cosin'"):
        mv.brute_force_knn(x, x, 3, "cosin")


def test_device_tensors_match_host():
    import torch

    b, q = data.gaussian_mixture_int(30_000, 128, 32, seed=8, nq=500)
    hids, hdist = mv.brute_force_knn(b, q, 10, "l2")
    tb, tq = torch.from_numpy(b).cuda(), torch.from_numpy(q).cuda()
    ids, dist = mv.brute_force_knn(tb, tq, 10, "l2")
    torch.cuda.synchronize()
    assert ids.is_cuda and ids.dtype == torch.int32
    assert np.array_equal(ids.cpu().numpy(), hids)
    assert np.array_equal(dist.cpu().numpy(), hdist)
    mv.synchronize()


def test_sharded_keys_merge_equals_single():
    # the multi-GPU path on one GPU: shards with id offsets, then merge_keys
    import torch

    b, q = data.gaussian_mixture_int(40_000, 128, 32, seed=12, nq=257)
    tb, tq = torch.from_numpy(b).cuda(), torch.from_numpy(q).cuda()
    bounds = [0, 9_999, 25_000, 40_000]
    lists = torch.stack([
        mv.knn_keys(tb[s:e], tq, 12, "l2", id_offset=s) for s, e in zip(bounds, bounds[1:])])
    ids, dist = mv.merge_keys(lists, 12, "l2", tq)
    oids, odist = O.brute_force_knn(b, q, 12, "l2")
    assert np.array_equal(ids.cpu().numpy(), oids)
    assert np.array_equal(dist.cpu().numpy(), odist)
    okeys = O.knn_keys(b, q, 12, "l2")
    full = mv.knn_keys(tb, tq, 12, "l2")
    assert np.array_equal(full.cpu().numpy().view(np.uint64), okeys)


def test_golden_fixtures():
    with open(os.path.join(os.path.dirname(__file__), "golden", "golden.json")) as f:
        cases = json.load(f)
    for case in cases:
        hamming, b, q = data.golden_inputs(case["input"])
        if hamming:
            ids, dist = mv.hamming_knn(b, q, case["k"])
        else:
            ids, dist = mv.brute_force_knn(b, q, case["k"], case["metric"])
        if case.get("exact", True):
            assert ids.tolist() == case["ids"], case["name"]
            assert dist.tolist() == case["distances"], case["name"]
        else:
            check_float(case["metric"], b, q, case["k"], ids, dist)


@pytest.mark.parametrize("metric,k", [("l2", 33), ("l2", 100), ("inner_product", 100),
                                      ("l2", 256), ("cosine", 64)])
def test_large_k_sampled_floor_path(metric, k):
    # k > 32 on a base large enough for the sampled-floor search (exact lists
    # of 4+ disjoint samples -> a floor, every candidate above it kept, the
    # best k selected); integer data bit-exact, unit rows within tolerance
    if metric == "cosine":
        b, q = data.lowrank_unit(80_000, 64, 16, seed=71, nq=300)
        ids, dist = mv.brute_force_knn(b, q, k, metric)
        check_float(metric, b, q, k, ids, dist)
        return
    b, q = data.gaussian_mixture_int(80_000, 128, 64, seed=72, nq=333)
    ids, dist = mv.brute_force_knn(b, q, k, metric)
    oids, odist = O.brute_force_knn(b, q, k, metric)
    assert np.array_equal(ids, oids)
    assert np.array_equal(dist, odist)


@pytest.mark.parametrize("n,d,k", [(140_000, 32, 64), (250_000, 32, 100), (600_000, 16, 256),
                                   (300_000, 32, 17), (700_000, 16, 100)])
def test_large_k_listed_floor_path(n, d, k):
    # k > 16 on a base of 64+ sampled tiles: the floor is the list kernel's
    # best 16 of every (6 k / 16)-th tile (the last two cases) or, where
    # that sample is too small, its best 32 of every (4 k / 32)-th tile;
    # integer data bit-exact
    import torch

    b, q = data.gaussian_mixture_int(n, d, 64, seed=73, nq=150)
    # device tensors: one search over the whole base (the host entry would
    # search a base this large in chunks)
    tids, tdist = mv.brute_force_knn(torch.from_numpy(b).cuda(), torch.from_numpy(q).cuda(), k,
                                     "l2")
    ids, dist = tids.cpu().numpy(), tdist.cpu().numpy()
    oids, odist = O.brute_force_knn(b, q, k, "l2")
    assert np.array_equal(ids, oids)
    assert np.array_equal(dist, odist)


@pytest.mark.parametrize("n,stride", [(200_000, 12), (610_000, 37)])
def test_large_k_listed_floor_underflow_falls_back(n, stride):
    # every near row sits in the sampled tiles (for k = 100 every 12th tile
    # with 32-key sample lists, every 37th with 16-key ones), so only the
    # sample's best kp clear its floor: the select step flags the queries
    # and the heap search gives the result
    import torch

    d, k = 16, 100
    rng = np.random.default_rng(74)
    b = np.full((n, d), 50.0, np.float32)
    tiles = (n + 255) // 256
    for t in range(0, tiles, stride):
        lo, hi = t * 256, min(n, t * 256 + 256)
        b[lo:hi] = rng.integers(0, 4, (hi - lo, d)).astype(np.float32)
    q = np.zeros((8, d), np.float32)
    mv.profile_enable(True)
    try:
        tids, tdist = mv.brute_force_knn(torch.from_numpy(b).cuda(), torch.from_numpy(q).cuda(),
                                         k, "l2")
        ids, dist = tids.cpu().numpy(), tdist.cpu().numpy()
        _, gemm_launches = mv.profile_read("gemm_topk")
        _, collect_launches = mv.profile_read("gemm_collect")
    finally:
        mv.profile_enable(False)
    assert collect_launches == 1 and gemm_launches == 2  # sample pass, then the heaps
    oids, odist = O.brute_force_knn(b, q, k, "l2")
    assert np.array_equal(ids, oids)
    assert np.array_equal(dist, odist)


def test_large_k_overflow_falls_back():
    # identical rows: every row ties the floor, the kept candidates overflow
    # their buffers and the search falls back to per-query heaps; the result
    # is still the lowest ids
    b = np.zeros((40_000, 32), np.float32)
    q = np.zeros((50, 32), np.float32)
    ids, dist = mv.brute_force_knn(b, q, 100, "l2")
    assert (ids == np.arange(100)[None, :]).all()
    assert (dist == 0).all()


@pytest.mark.parametrize("metric,k", [("l2", 10), ("inner_product", 1), ("cosine", 10),
                                      ("cosine", 50), ("l2", 128)])
def test_inexact_floats_one_pass_with_rescoring(metric, k):
    # general float32 rows on a base of 64+ tiles: one fp16 pass keeps every
    # candidate within its error bound of a sampled floor, exact float32
    # scores decide (recall 1, distances within 1e-4)
    b, q = data.lowrank_unit(70_000, 256, 32, seed=81, nq=400)
    if metric != "cosine":
        b = b * np.float32(3.7)
        q = q * np.float32(0.6)
    ids, dist = mv.brute_force_knn(b, q, k, metric)
    check_float(metric, b, q, k, ids, dist)


def test_inexact_floats_near_ties():
    # rows that differ by far less than the fp16 rounding: the margin keeps
    # them all, the exact scores order them
    rng = np.random.default_rng(82)
    b = data.normal_rows(40_000, 64, seed=83)
    b[20_000:] = b[:20_000] + rng.standard_normal((20_000, 64)).astype(np.float32) * 1e-5
    q = b[:300] + rng.standard_normal((300, 64)).astype(np.float32) * 1e-3
    ids, dist = mv.brute_force_knn(b, q, 10, "l2")
    check_float("l2", b, q, 10, ids, dist)


@pytest.mark.parametrize("metric,k,integer", [("l2", 10, True), ("inner_product", 20, True),
                                              ("cosine", 10, False)])
def test_host_api_chunked_copy(metric, k, integer):
    # host buffers of 2^18+ rows: the base is copied in chunks, each searched
    # as it lands, and the chunks' lists merged; the results equal the
    # device-pointer search (bit for bit on integer data)
    import torch

    if integer:
        b, q = data.gaussian_mixture_int(300_001, 64, 64, seed=91, nq=500)
    else:
        b, q = data.lowrank_unit(300_001, 64, 16, seed=92, nq=500)
    ids, dist = mv.brute_force_knn(b, q, k, metric)
    dids, ddist = mv.brute_force_knn(torch.from_numpy(b).cuda(), torch.from_numpy(q).cuda(), k,
                                     metric)
    torch.cuda.synchronize()
    if integer:
        assert np.array_equal(ids, dids.cpu().numpy())
        assert np.array_equal(dist, ddist.cpu().numpy())
        oids, odist = O.brute_force_knn(b, q, k, metric)
        assert np.array_equal(ids, oids) and np.array_equal(dist, odist)
    else:
        check_float(metric, b, q, k, ids, dist)
