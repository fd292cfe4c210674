"""GPU parity of the row-wise selection entries against the CPU oracle:
topk_merge (one merge step, src/knn.cpp:37-69 and src/kernels.h:37-229) and
refine (exact re-ranking, src/ivf.cpp:1642-1708).  Selection is bit-exact
(ids and scores); refine's distances are bit-exact on integer data and
within 1e-4 on float data (the sums run in another order)."""

import numpy as np
import pytest

import mlxvs_b200 as mv
from oracle import oracle as O
from tests import data

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("k,t", [(1, 1000), (10, 65536), (100, 3000), (256, 5000), (64, 10)])
def test_topk_merge_first_and_running(k, t):
    rng = np.random.default_rng(k + t)
    nq = 37
    s = rng.integers(-50, 50, (nq, t)).astype(np.float32)  # many ties
    s[0, : min(t, 5)] = -np.inf
    ids0, sc0 = mv.topk_merge(s, None, None, 1000, True, k)
    oids0, osc0 = O.topk_merge(s, None, None, 1000, True, k)
    assert np.array_equal(ids0, oids0) and np.array_equal(sc0, osc0)
    s2 = rng.standard_normal((nq, t)).astype(np.float32)
    ids1, sc1 = mv.topk_merge(s2, ids0, sc0, -3, False, k)
    oids1, osc1 = O.topk_merge(s2, oids0, osc0, -3, False, k)
    assert np.array_equal(ids1, oids1) and np.array_equal(sc1, osc1)


def test_topk_merge_device_tensors_and_errors():
    import torch

    rng = np.random.default_rng(5)
    s = rng.standard_normal((300, 777)).astype(np.float32)
    want = mv.topk_merge(s, None, None, 0, True, 33)
    ids, sc = mv.topk_merge(torch.from_numpy(s).cuda(), None, None, 0, True, 33)
    torch.cuda.synchronize()
    assert np.array_equal(ids.cpu().numpy(), want[0])
    assert np.array_equal(sc.cpu().numpy(), want[1])
    with pytest.raises(ValueError, match="k must be in"):
        mv.topk_merge(s, None, None, 0, True, 257)
    with pytest.raises(ValueError, match="float32"):
        mv.topk_merge(s.astype(np.float64), None, None, 0, True, 3)


@pytest.mark.parametrize("metric", ["l2", "inner_product"])
def test_refine_integer_bit_exact(metric):
    x, q = data.gaussian_mixture_int(50_000, 128, 32, seed=61, nq=500)
    rng = np.random.default_rng(62)
    cand = rng.integers(-10, 50_010, (500, 40))
    cand[:, 5] = cand[:, 4]  # repeated candidates are both kept
    ids, dist = mv.refine(x, q, cand, 10, metric)
    oids, odist = O.refine(x, q, cand, 10, metric)
    assert np.array_equal(ids, oids)
    assert np.array_equal(dist, odist)


@pytest.mark.parametrize("metric", ["l2", "cosine", "inner_product"])
def test_refine_float_tolerance(metric):
    x = data.normal_rows(20_000, 96, seed=63)
    q = data.normal_rows(200, 96, seed=64)
    # candidates: the exact neighbours shuffled among other rows
    scores = data.exact_scores(metric, q, x)
    top = np.argsort(-scores, axis=1)[:, :20]
    rng = np.random.default_rng(65)
    others = [rng.choice(np.setdiff1d(np.arange(20_000), top[i]), 60, replace=False)
              for i in range(200)]
    cand = np.concatenate([top, np.stack(others)], 1)
    cand = np.take_along_axis(cand, rng.permuted(np.tile(np.arange(80), (200, 1)), axis=1), 1)
    ids, dist = mv.refine(x, q, cand, 20, metric)
    assert data.recall(ids, scores, 20, tol=1e-4) == 1.0
    want = np.take_along_axis(scores, ids.astype(np.int64), 1)
    want = -want if metric == "l2" else want
    assert np.allclose(dist, want, rtol=1e-4, atol=1e-4)


def test_refine_device_missing_and_errors():
    import torch

    x, q = data.gaussian_mixture_int(5_000, 32, 8, seed=66, nq=64)
    cand = np.full((64, 12), -1, np.int64)
    cand[:, :5] = np.arange(5)
    cand[:, 5] = 10**9  # outside the dataset: skipped
    hids, hdist = mv.refine(x, q, cand, 8, "l2")
    assert (hids[:, 5:] == -1).all() and np.isposinf(hdist[:, 5:]).all()
    oids, odist = O.refine(x, q, cand, 8, "l2")
    assert np.array_equal(hids, oids) and np.array_equal(hdist, odist)
    ids, dist = mv.refine(torch.from_numpy(x).cuda(), torch.from_numpy(q).cuda(),
                          torch.from_numpy(cand).cuda(), 8, "l2")
    torch.cuda.synchronize()
    assert np.array_equal(ids.cpu().numpy(), hids)
    assert np.array_equal(dist.cpu().numpy(), hdist)
    with pytest.raises(ValueError, match="candidates per query"):
        mv.refine(x, q, cand, 13, "l2")
    with pytest.raises(ValueError, match="must match"):
        mv.refine(x, q[:, :5], cand, 3, "l2")
    mv.synchronize()


@pytest.mark.parametrize("order", ["random", "best_first", "worst_first", "mixed"])
@pytest.mark.parametrize("k,lists,nq", [(1, 7, 45), (4, 30, 100), (5, 2, 33), (10, 13, 10_000),
                                        (10, 19, 77), (10, 20, 70), (16, 12, 64), (17, 5, 31),
                                        (32, 6, 50), (32, 7, 40), (32, 24, 20), (1, 40, 64),
                                        (10, 40, 50)])
def test_merge_keys_duplicates_and_empty_slots(k, lists, nq, order):
    # the candidate lists of the units or ranks of one search: a key may sit
    # in several lists (units start from an earlier unit's list), slots may
    # be empty (0); lists come best first (merged lists), worst first with
    # the empty slots in front (the fused kernel's register lists) or in no
    # order (its heaps).  Up to 768 candidates in up to 32 lists per query
    # take the four-lanes-per-query merge, more lists the warp-per-query one.
    torch = pytest.importorskip("torch")
    rng = np.random.default_rng(1000 * k + lists)
    table = rng.integers(-40, 40, size=(nq, 300)).astype(np.float32)
    if order == "random":  # ids may repeat inside a list too
        ids = rng.integers(0, 300, size=(lists, nq, k))
    else:
        ids = np.argsort(rng.random((lists, nq, 300)), axis=2)[..., :k]
    scores = np.take_along_axis(table[None].repeat(lists, 0), ids, axis=2)
    keys = (O._order_bits(scores).astype(np.uint64) << np.uint64(32)) | \
        (~ids.astype(np.uint32)).astype(np.uint64)
    keys[rng.random(keys.shape) < 0.2] = 0
    if order in ("best_first", "mixed"):
        srt = np.sort(keys, axis=2)[..., ::-1]
        if order == "mixed":
            pick = rng.random(nq) < 0.5
            keys[:, pick, :] = srt[:, pick, :]
        else:
            keys = srt.copy()
    elif order == "worst_first":
        keys = np.sort(keys, axis=2)
    # expected: the k largest distinct non-zero keys per query, best first
    okeys = np.zeros((nq, k), np.uint64)
    for i in range(nq):
        u = np.unique(keys[:, i, :])[::-1]
        u = u[u != 0][:k]
        okeys[i, :len(u)] = u
    oids, oscores = O.decode_keys(okeys)
    t = torch.from_numpy(keys.copy().view(np.int64)).cuda()
    gids, gdist = mv.merge_keys(t, k, "inner_product")
    assert np.array_equal(gids.cpu().numpy(), oids)
    assert np.array_equal(gdist.cpu().numpy(), oscores)


@pytest.mark.parametrize("lists", [6, 40])
def test_merge_keys_l2_distances(lists):
    # L2 distances max(|q|^2 - score, 0) of merged keys: up to 32 lists the
    # merge kernel computes |q|^2 itself, past that a separate pass does
    torch = pytest.importorskip("torch")
    k, nq, d = 10, 1000, 37
    rng = np.random.default_rng(lists)
    q = rng.integers(0, 256, size=(nq, d)).astype(np.float32)
    ids = np.argsort(rng.random((lists, nq, 500)), axis=2)[..., :k]
    scores = rng.integers(0, 2 ** 20, size=(lists, nq, k)).astype(np.float32)
    keys = (O._order_bits(scores).astype(np.uint64) << np.uint64(32)) | \
        (~ids.astype(np.uint32)).astype(np.uint64)
    keys = np.sort(keys, axis=2)[..., ::-1].copy()
    best = np.sort(keys.transpose(1, 0, 2).reshape(nq, -1), axis=1)[:, ::-1][:, :k]
    oids, oscores = O.decode_keys(best)
    qn = (q.astype(np.float64) ** 2).sum(1).astype(np.float32)  # exact: integers < 2^24
    odist = np.maximum(qn[:, None] - oscores, 0).astype(np.float32)
    t = torch.from_numpy(keys.view(np.int64)).cuda()
    gids, gdist = mv.merge_keys(t, k, "l2", torch.from_numpy(q).cuda())
    assert np.array_equal(gids.cpu().numpy(), oids)
    assert np.array_equal(gdist.cpu().numpy(), odist)
