"""GPU parity of hamming_knn (C API, sm_100a popcount kernel) against the
CPU oracle: ids and distances bit-exact, ties to the lower id."""

import numpy as np
import pytest

import mlxvs_b200 as mv
from oracle import oracle as O
from tests import data

pytestmark = pytest.mark.gpu


def test_tiny_kat():
    # python/tests/test_cuvs.py:844-849
    codes = np.array([[0b1111, 0], [0b1, 0]], dtype=np.uint8)
    ids, dist = mv.hamming_knn(codes, codes[:1], 2)
    assert ids[0].tolist() == [0, 1]
    assert dist[0].tolist() == [0.0, 3.0]


@pytest.mark.parametrize("nbytes", [1, 5, 16, 32, 48, 128, 130, 256, 512])
def test_clustered_codes_bit_exact(nbytes):
    # tests/test_ivf.cpp:252-311 generator shape (40 prototypes, 10% flips)
    rows, q = data.hamming_codes(20_000 + 3, nbytes, 40, 0.1, seed=7, nq=300)
    ids, dist = mv.hamming_knn(rows, q, 10)
    oids, odist = O.hamming_knn(rows, q, 10)
    assert np.array_equal(ids, oids)
    assert np.array_equal(dist, odist)


@pytest.mark.parametrize("k", [1, 10, 64, 100, 256])
def test_k_sweep(k):
    rows, q = data.hamming_codes(30_000, 128, 4096, 0.1, seed=11, nq=200)
    ids, dist = mv.hamming_knn(rows, q, k)
    oids, odist = O.hamming_knn(rows, q, k)
    assert np.array_equal(ids, oids)
    assert np.array_equal(dist, odist)


def test_many_ties():
    # few distinct codes: distances tie massively, lower ids must win
    rng = np.random.default_rng(3)
    protos = rng.integers(0, 256, (4, 32), dtype=np.uint8)
    rows = protos[rng.integers(0, 4, 50_000)]
    q = protos[rng.integers(0, 4, 64)]
    ids, dist = mv.hamming_knn(rows, q, 20)
    oids, odist = O.hamming_knn(rows, q, 20)
    assert np.array_equal(ids, oids)
    assert np.array_equal(dist, odist)
    for _ in range(5):
        again, _ = mv.hamming_knn(rows, q, 20)
        assert np.array_equal(again, ids)


def test_fewer_rows_than_k_and_empty():
    rows, q = data.hamming_codes(5, 16, 2, 0.1, seed=1, nq=3)
    ids, dist = mv.hamming_knn(rows, q, 8)
    assert (ids[:, :5] >= 0).all() and (ids[:, 5:] == -1).all()
    assert np.isposinf(dist[:, 5:]).all()
    ids, dist = mv.hamming_knn(rows[:0], q, 4)
    assert (ids == -1).all() and np.isposinf(dist).all()
    ids, _ = mv.hamming_knn(rows, q[:0], 4)
    assert ids.shape == (0, 4)


def test_errors():
    rows, q = data.hamming_codes(10, 16, 2, 0.1, seed=1, nq=3)
    with pytest.raises(ValueError):
        mv.hamming_knn(rows, q, 300)
    with pytest.raises(ValueError):
        mv.hamming_knn(rows.astype(np.int32), q, 3)
    with pytest.raises(ValueError):
        mv.hamming_knn(rows, q[:, :8], 3)


def test_device_and_sharded():
    import torch

    rows, q = data.hamming_codes(50_000, 128, 4096, 0.1, seed=5, nq=333)
    oids, odist = O.hamming_knn(rows, q, 10)
    tr, tq = torch.from_numpy(rows).cuda(), torch.from_numpy(q).cuda()
    ids, dist = mv.hamming_knn(tr, tq, 10)
    assert np.array_equal(ids.cpu().numpy(), oids)
    assert np.array_equal(dist.cpu().numpy(), odist)
    bounds = [0, 12_345, 30_000, 50_000]
    lists = torch.stack([
        mv.hamming_keys(tr[s:e], tq, 10, id_offset=s) for s, e in zip(bounds, bounds[1:])])
    ids, dist = mv.merge_keys(lists, 10, "hamming")
    assert np.array_equal(ids.cpu().numpy(), oids)
    assert np.array_equal(dist.cpu().numpy(), odist)
    mv.synchronize()


def test_host_api_chunked_copy():
    # 2^18+ codes from host memory: copied in chunks, each searched as it
    # lands, the lists merged; bit-exact with the device entry and the oracle
    import torch

    rows, q = data.hamming_codes(300_001, 64, 1024, 0.1, seed=95, nq=300)
    ids, dist = mv.hamming_knn(rows, q, 10)
    dids, ddist = mv.hamming_knn(torch.from_numpy(rows).cuda(), torch.from_numpy(q).cuda(), 10)
    torch.cuda.synchronize()
    assert np.array_equal(ids, dids.cpu().numpy())
    assert np.array_equal(dist, ddist.cpu().numpy())
    oids, odist = O.hamming_knn(rows, q, 10)
    assert np.array_equal(ids, oids) and np.array_equal(dist, odist)
