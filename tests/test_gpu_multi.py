"""The row-sharded search on 2 GPUs of one node (NCCL, one process per GPU):
results equal the single-GPU search (bit for bit on integer data, recall 1
on float data, where each shard's operand scale may round a score
differently).  The 2-GPU test is skipped on a box with fewer GPUs; the
stream= test runs on one."""

import os
import socket
from datetime import timedelta

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from tests import data

pytestmark = [pytest.mark.gpu, pytest.mark.timeout(600)]

WORLD = 2


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


CASES = [("l2", 10, True), ("l2", 10, False), ("inner_product", 12, False), ("l2", 64, False)]


def make_case(metric, integer):
    if integer:
        return data.gaussian_mixture_int(60_000, 128, 32, seed=41, nq=1_000)
    b = data.normal_rows(60_000, 128, seed=42)
    q = data.normal_rows(1_000, 128, seed=43)
    b[:20_000] *= np.float32(2.5)  # the shards' operand scales differ
    return b, q


def _worker(rank, world, port, out):
    import mlxvs_b200 as mv
    from mlxvs_b200 import distributed as mvd

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=timedelta(seconds=60), device_id=dev)
    try:
        for metric, k, integer in CASES:
            b, q = make_case(metric, integer)
            bounds = mvd.shard_bounds(b.shape[0], world)
            lo, hi = bounds[rank], bounds[rank + 1]
            shard = torch.from_numpy(b[lo:hi]).to(dev)
            tq = torch.from_numpy(q).to(dev)
            first = mvd.sharded_brute_force_knn(shard, tq, k, metric, id_offset=lo)
            ids, dist_ = mvd.sharded_brute_force_knn(shard, tq, k, metric, id_offset=lo)
            mv.synchronize()
            # every rank holds the same result, the same on every call
            same = bool(torch.equal(ids, first[0]) and torch.equal(dist_, first[1]))
            gathered = [torch.empty_like(ids) for _ in range(world)]
            dist.all_gather(gathered, ids)
            same = same and all(bool(torch.equal(g, ids)) for g in gathered)
            single = None
            if rank == 0:
                sids, sdist = mv.brute_force_knn(torch.from_numpy(b).to(dev), tq, k, metric)
                if integer:
                    single = bool(torch.equal(ids, sids) and torch.equal(dist_, sdist))
                else:
                    scores = data.exact_scores(metric, q, b)
                    single = data.recall(ids.cpu().numpy(), scores, k, tol=1e-4) == 1.0
            out[(rank, metric, k, integer)] = (same, single)
        # stream=: a side stream kept busy first, so a gather queued on
        # another stream would read keys that are not written yet
        b, q = make_case("l2", True)
        bounds = mvd.shard_bounds(b.shape[0], world)
        lo, hi = bounds[rank], bounds[rank + 1]
        shard = torch.from_numpy(b[lo:hi]).to(dev)
        tq = torch.from_numpy(q).to(dev)
        want = mvd.sharded_brute_force_knn(shard, tq, 10, "l2", id_offset=lo)
        side = torch.cuda.Stream(device=dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            torch.cuda._sleep(200_000_000)
        got = mvd.sharded_brute_force_knn(shard, tq, 10, "l2", id_offset=lo, stream=side)
        side.synchronize()
        out[(rank, "stream")] = bool(torch.equal(got[0], want[0]) and
                                     torch.equal(got[1], want[1]))
        # the peer exchange (lists read from the other GPU's memory) gives
        # the NCCL path's results, step after step (the two key slots
        # alternate), also for a step with no queries and for Hamming codes
        ex = mvd.PeerExchange(1_000 * 32)
        okx = True
        for metric, k, integer in CASES:
            if not ex.fits(1_000, k):
                continue
            b, q = make_case(metric, integer)
            bounds = mvd.shard_bounds(b.shape[0], world)
            lo, hi = bounds[rank], bounds[rank + 1]
            shard = torch.from_numpy(b[lo:hi]).to(dev)
            tq = torch.from_numpy(q).to(dev)
            want = mvd.sharded_brute_force_knn(shard, tq, k, metric, id_offset=lo)
            for _ in range(3):
                got = mvd.sharded_brute_force_knn(shard, tq, k, metric, id_offset=lo, exchange=ex)
                okx &= bool(torch.equal(got[0], want[0]) and torch.equal(got[1], want[1]))
            empty = mvd.sharded_brute_force_knn(shard, tq[:0], k, metric, id_offset=lo,
                                                exchange=ex)
            okx &= tuple(empty[0].shape) == (0, k)
        codes, qc = data.hamming_codes(40_000, 128, 64, 0.1, seed=45, nq=500)
        bounds = mvd.shard_bounds(codes.shape[0], world)
        lo, hi = bounds[rank], bounds[rank + 1]
        tcodes = torch.from_numpy(codes[lo:hi]).to(dev)
        tqc = torch.from_numpy(qc).to(dev)
        want = mvd.sharded_hamming_knn(tcodes, tqc, 10, id_offset=lo)
        got = mvd.sharded_hamming_knn(tcodes, tqc, 10, id_offset=lo, exchange=ex)
        okx &= bool(torch.equal(got[0], want[0]) and torch.equal(got[1], want[1]))
        mv.synchronize()
        torch.cuda.synchronize()
        dist.barrier()
        ex.close()
        out[(rank, "exchange")] = okx
        # the k-NN graph split by rows (all rows on every rank, no exchange
        # but the final gather)
        x, _ = data.gaussian_mixture_int(20_001, 64, 16, seed=44)
        tx = torch.from_numpy(x).to(dev)
        gids, gdist = mvd.sharded_all_neighbors(tx, 16, "l2")
        sids, sdist = mv.all_neighbors(tx, 16, "l2", algo="brute_force")
        out[(rank, "allnn")] = bool(torch.equal(gids, sids) and torch.equal(gdist, sdist))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < WORLD,
                    reason="needs 2 GPUs")
def test_two_gpus_match_single():
    port = free_port()
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        out = mgr.dict()
        mp.start_processes(_worker, args=(WORLD, port, out), nprocs=WORLD, start_method="spawn",
                           join=True)
        res = dict(out)
    for metric, k, integer in CASES:
        for r in range(WORLD):
            same, single = res[(r, metric, k, integer)]
            assert same, (r, metric, k, integer)
            if r == 0:
                assert single, (metric, k, integer)
    for r in range(WORLD):
        assert res[(r, "allnn")], r
        assert res[(r, "stream")], r
        assert res[(r, "exchange")], r


@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")
def test_stream_argument_one_rank():
    # stream= carries the search and its merge (world size 1 here: no
    # process group, the gather is the rank's own keys)
    import mlxvs_b200 as mv
    from mlxvs_b200 import distributed as mvd

    dev = torch.device("cuda", 0)
    b, q = make_case("l2", True)
    tb, tq = torch.from_numpy(b).to(dev), torch.from_numpy(q).to(dev)
    want = mv.brute_force_knn(tb, tq, 10, "l2")
    side = torch.cuda.Stream(device=dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        torch.cuda._sleep(100_000_000)
    ids, dst = mvd.sharded_brute_force_knn(tb, tq, 10, "l2", id_offset=0, stream=side)
    side.synchronize()
    assert torch.equal(ids, want[0]) and torch.equal(dst, want[1])
    # a raw cudaStream_t handle works the same way
    ids2, dst2 = mvd.sharded_brute_force_knn(tb, tq, 10, "l2", id_offset=0,
                                             stream=side.cuda_stream)
    side.synchronize()
    assert torch.equal(ids2, want[0]) and torch.equal(dst2, want[1])


@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")
def test_peer_exchange_one_rank():
    # the exchange's kernels with one GPU (no process group): the wait sees
    # this GPU's own flag, the merge reads this GPU's slot; several epochs
    # (both slots), sizes and kinds, against the plain search
    import mlxvs_b200 as mv
    from mlxvs_b200 import distributed as mvd

    dev = torch.device("cuda", 0)
    b, _ = data.gaussian_mixture_int(50_000, 128, 32, seed=46)
    tb = torch.from_numpy(b).to(dev)
    ex = mvd.PeerExchange(2_000 * 32)
    try:
        for i, (nq, k, metric) in enumerate([(700, 10, "l2"), (2_000, 32, "inner_product"),
                                             (0, 10, "l2"), (1_999, 16, "l2")]):
            _, q = data.gaussian_mixture_int(10, 128, 32, seed=50 + i, nq=max(nq, 1))
            tq = torch.from_numpy(q[:nq]).to(dev)
            ids, dst = mvd.sharded_brute_force_knn(tb, tq, k, metric, id_offset=0, exchange=ex)
            want = mv.brute_force_knn(tb, tq, k, metric)
            assert torch.equal(ids, want[0]) and torch.equal(dst, want[1]), (nq, k, metric)
            assert ex.epoch == i + 1
        assert not ex.fits(2_000, 33) and not ex.fits(3_000, 32)
        codes, qc = data.hamming_codes(20_000, 64, 32, 0.1, seed=47, nq=300)
        got = mvd.sharded_hamming_knn(torch.from_numpy(codes).to(dev),
                                      torch.from_numpy(qc).to(dev), 10, id_offset=0, exchange=ex)
        want = mv.hamming_knn(codes, qc, 10)
        assert np.array_equal(got[0].cpu().numpy(), want[0])
        assert np.array_equal(got[1].cpu().numpy(), want[1])
        mv.synchronize()
    finally:
        ex.close()
