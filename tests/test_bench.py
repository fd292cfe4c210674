"""bench.py's host-side pieces, without a GPU: the workload table, the
line's config keys, the committed DRAM-traffic captures the roofline reads,
the peaks, and the reference arm (the oracle on the host cores) on the
smallest configuration."""

import argparse
import io
import json
import os
import sys
from contextlib import redirect_stdout

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import bench  # noqa: E402


def test_workloads_are_complete():
    for name, w in bench.WORKLOADS.items():
        for key in ("kind", "n", "nq", "k", "desc"):
            assert key in w, (name, key)
        assert w["kind"] in ("knn", "knn-unit", "allnn", "hamming", "topk", "refine"), name
        if w["kind"] in ("knn", "knn-unit", "allnn", "refine"):
            assert w["d"] >= 1 and w["metric"] in ("l2", "inner_product", "cosine"), name
        if w["kind"] == "hamming":
            assert w["bytes"] % 16 == 0, name
    assert bench.DEFAULT_WORKLOAD == "knn-l2-1m-k10"
    w = bench.WORKLOADS[bench.DEFAULT_WORKLOAD]
    assert (w["n"], w["nq"], w["d"], w["k"], w["metric"]) == (1_000_000, 10_000, 128, 10, "l2")


def test_config_names_the_workload_and_its_sizes():
    args = argparse.Namespace(workload=bench.DEFAULT_WORKLOAD, shard_of=1, exchange="peer",
                              entry="default")
    w = bench.WORKLOADS[bench.DEFAULT_WORKLOAD]
    for world in (1, 2, 8):
        cfg = bench.config_of(args, w, world)
        assert cfg["workload"] == bench.DEFAULT_WORKLOAD
        assert (cfg["n"], cfg["queries"], cfg["k"]) == (w["n"], w["nq"], w["k"])
        assert ("exchange" in cfg) == (world > 1)


def test_traffic_captures_cover_the_default_workload_at_every_world_size():
    with open(bench.TRAFFIC_FILE) as f:
        table = json.load(f)
    algorithmic = 1_000_000 * (128 * 2 + 32)  # fp16 rows + |b|^2 pieces
    for world in (1, 2, 4, 8):
        b, src = bench.load_traffic(bench.DEFAULT_WORKLOAD, world)
        assert b is not None and "ncu" in src, world
        # a rank's DRAM bytes: at least its share of the algorithmic bytes,
        # and not wildly above it
        share = algorithmic / world
        assert 0.9 * share < b < 2.0 * share, (world, b)
    for key, e in table.items():
        assert e["bytes_per_launch"] > 0 and e["source"].startswith("ncu "), key
    assert bench.load_traffic("no-such-workload", 1)[0] is None


def test_peaks_are_positive():
    p = bench.load_peaks()
    assert p["hbm_gbs"] > 0 and p["bf16"] > 0 and p["bf16_sustained"] > 0
    assert p["source"] in ("measured", "fallback")


def test_reference_arm_runs_on_the_host():
    pytest.importorskip("numpy")
    from oracle import oracle as O

    O.build()
    args = argparse.Namespace(workload="knn-l2-100k-k10", gpus=1, steps=1, warmup=1,
                              impl="reference", shard_of=1, exchange="peer", entry="default")
    buf = io.StringIO()
    with redirect_stdout(buf):
        rc = bench.reference_arm(args, bench.WORKLOADS[args.workload], bench.load_peaks())
    assert rc == 0
    line = json.loads(buf.getvalue().strip().splitlines()[-1])
    assert line["impl"] == "reference" and line["value"] > 0
    assert line["cpu_baseline"]["cores"] >= 1 and line["cpu_baseline"]["kind"] == "port"
    assert line["e2e"]["h2d_bytes_per_step"] == 0
    assert line["config"]["workload"] == "knn-l2-100k-k10"
