"""The row-sharded path's host logic on CPU ranks (gloo, world size 2): shard
bounds, the all-gather of per-rank key lists, and their merge reproduce the
single-process result; a rank that never reaches the exchange is detected by
the others through the process group's timeout, not by a hang."""

import os
import socket
from datetime import timedelta

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from mlxvs_b200 import distributed as mvd
from oracle import oracle as O
from tests import data


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port, timeout_s):
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=timedelta(seconds=timeout_s))


def _sharded_worker(rank, world, port, k, out):
    _init(rank, world, port, 60)
    try:
        b, q = data.gaussian_mixture_int(5_000, 32, 8, seed=3, nq=40)
        bounds = mvd.shard_bounds(b.shape[0], world)
        lo, hi = bounds[rank], bounds[rank + 1]
        # the CPU oracle stands in for the per-rank kernel (mlxvs_knn_keys_device)
        keys = O.knn_keys(b[lo:hi], q, k, "l2", id_offset=lo)
        lists = mvd.gather_lists(torch.from_numpy(keys.view(np.int64)))
        merged = O.merge_keys(lists.numpy().view(np.uint64), k)
        out[rank] = merged.tobytes()
    finally:
        dist.destroy_process_group()


def test_shard_bounds():
    assert mvd.shard_bounds(10, 3) == [0, 3, 6, 10]
    assert mvd.shard_bounds(1_000_000, 8)[1] == 125_000
    assert mvd.shard_bounds(5, 8)[-1] == 5


def test_gloo_world2_matches_single():
    world, k = 2, 12
    port = free_port()
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        out = mgr.dict()
        mp.start_processes(_sharded_worker, args=(world, port, k, out), nprocs=world,
                           start_method="spawn", join=True)
        results = [np.frombuffer(out[r], np.uint64).reshape(-1, k) for r in range(world)]
    b, q = data.gaussian_mixture_int(5_000, 32, 8, seed=3, nq=40)
    full = O.knn_keys(b, q, k, "l2")
    for r in results:
        assert np.array_equal(r, full)


def _dropout_worker(rank, world, port, out):
    _init(rank, world, port, 5)
    try:
        if rank == 1:
            out[1] = "left before the exchange"
            return  # never joins the all-gather
        keys = torch.zeros((4, 3), dtype=torch.int64)
        try:
            mvd.gather_lists(keys)
            out[0] = "no error"
        except Exception as e:  # the process group's timeout
            out[0] = "error: " + type(e).__name__
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


@pytest.mark.timeout(120)
def test_missing_rank_is_reported_not_hung():
    port = free_port()
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        out = mgr.dict()
        mp.start_processes(_dropout_worker, args=(2, port, out), nprocs=2, start_method="spawn",
                           join=True)
        assert out[1] == "left before the exchange"
        assert out[0].startswith("error"), out[0]
