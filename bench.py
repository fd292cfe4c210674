#!/usr/bin/env python
"""Exact k-NN benchmark (BASELINE.json's metric: queries/s on 1M x 128 fp32,
L2, k=10, 10k queries; base rows sharded across the GPUs of one node).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME]
    python bench.py --impl reference ...    (the CPU reference arm)
    torchrun --nproc-per-node N bench.py --gpus N ...

A step is one exact search of every query against the whole base: the
fp32 -> fp16 input conversion, the fused tcgen05 distance + top-k kernel,
(for N > 1) the exchange of each rank's [nq, k] candidates (read from the
peers' memory over NVLink; `--exchange nccl` for an NCCL all-gather), and
the merge to ids and distances.  The topk-merge and refine workloads time
those two callers of the search on one GPU against HBM bandwidth.  `value` is whole-job queries/s with the inputs
resident in HBM, L2 flushed before every timed step (a rank's shard is
smaller than L2 at 8 GPUs); `e2e` is the same through the host-memory API,
copies included.
Inputs are seeded synthetic data with BASELINE's distributions.
"""

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

WORKLOADS = {
    # BASELINE config 1 (the headline): 1M x 128 integer-valued fp32, L2
    "knn-l2-1m-k10": dict(kind="knn", n=1_000_000, nq=10_000, d=128, k=10, metric="l2",
                          clusters=1024,
                          desc="exact L2 k-NN, base 1M x 128 fp32 (integer-valued Gaussian "
                               "mixture, 1024 clusters), 10k queries, k=10"),
    "knn-l2-1m-k100": dict(kind="knn", n=1_000_000, nq=10_000, d=128, k=100, metric="l2",
                           clusters=1024, desc="config 1 with k=100"),
    # BASELINE config 0
    "knn-l2-100k-k10": dict(kind="knn", n=100_000, nq=1_000, d=128, k=10, metric="l2",
                            clusters=64, desc="config 0: 100k x 128, 1k queries, k=10"),
    # BASELINE config 2 (cosine, unit rows with a shared rank-64 part)
    "knn-cos-1m-1536": dict(kind="knn-unit", n=1_000_000, nq=10_000, d=1536, k=10,
                            metric="cosine", rank=64,
                            desc="config 2: 1M x 1536 fp32 unit rows, cosine, k=10"),
    # config 2 at a fifth of the rows: the profiling case (a few GB on the
    # device, still far larger than L2)
    "knn-cos-200k-1536": dict(kind="knn-unit", n=200_000, nq=10_000, d=1536, k=10,
                              metric="cosine", rank=64,
                              desc="config 2 at 200k x 1536 unit rows, cosine, k=10"),
    # config 2 with float16 storage (the rows rounded to fp16, computed in
    # fp32 after the upcast, as the reference does with an f16 array)
    "knn-cos-1m-1536-f16": dict(kind="knn-unit", n=1_000_000, nq=10_000, d=1536, k=10,
                                metric="cosine", rank=64, f16=True,
                                desc="config 2 with float16 storage: 1M x 1536 unit rows "
                                     "rounded to fp16, cosine, k=10"),
    # the exact k-NN graph (all_neighbors, one cluster,
    # brute force) of the config-1 generator's 1M rows, k=32 (the reference
    # searches k + 1 = 33 and drops each row itself)
    "allnn-l2-1m-k32": dict(kind="allnn", n=1_000_000, nq=1_000_000, d=128, k=32, metric="l2",
                            clusters=1024,
                            desc="config 3: all_neighbors of 1M x 128 fp32 (integer-valued "
                                 "mixture), L2, k=32 self excluded"),
    # config 4's codes at a tenth of the rows: the profiling case (its
    # unpacked rows, 1 GB, keep an ncu capture small)
    "hamming-1m-1024b": dict(kind="hamming", n=1_000_000, nq=10_000, bytes=128, k=10,
                             prototypes=4096, flip=0.1,
                             desc="config 4 at 1M x 1024-bit codes, 10k queries, k=10"),
    # BASELINE config 4
    "hamming-10m-1024b": dict(kind="hamming", n=10_000_000, nq=10_000, bytes=128, k=10,
                              prototypes=4096, flip=0.1,
                              desc="config 4: 10M x 1024-bit codes, 10k queries, k=10"),
    # the callers either side of the search (not BASELINE configurations):
    # one topk_merge step over 10k rows of 16,384 scores (655 MB, read once),
    # and refine of 1,024 candidates per query over config 1's rows
    "topk-merge-10k-t16384-k100": dict(kind="topk", n=16_384, nq=10_000, k=100,
                                       desc="topk_merge: 10k rows x 16,384 integer-valued "
                                            "float32 scores, k=100, first step"),
    "refine-10k-c1024-k10": dict(kind="refine", n=1_000_000, nq=10_000, d=128, c=1024, k=10,
                                 metric="l2", clusters=1024,
                                 desc="refine: 10k queries x 1,024 random candidate rows of "
                                      "config 1's 1M x 128 base, L2, k=10"),
}
DEFAULT_WORKLOAD = "knn-l2-1m-k10"
# twice the B200's 126 MB L2
FLUSH_BYTES = 256 << 20
METRIC = "exact k-NN queries/s (1M×128 fp32, k=10) at 1/2/4/8 B200; % tensor-pipe roofline"

# DRAM bytes per launch of the dominant kernel, measured by ncu for the
# exact kernel variant and the per-rank work of each world size (a rank's
# shard emulated on one GPU with --shard-of N): profiles/traffic.json, keyed
# "workload@N", each entry with the command that produced it.
TRAFFIC_FILE = os.path.join(ROOT, "profiles", "traffic.json")


def load_traffic(workload, world):
    try:
        with open(TRAFFIC_FILE) as f:
            table = json.load(f)
    except (OSError, ValueError):
        return None, "no capture"
    e = table.get(f"{workload}@{world}")
    if not e:
        return None, f"no capture of {workload} at N={world}"
    return e["bytes_per_launch"], e.get("source", "ncu")


def host_threads():
    """Host cores this process may run on (torchrun's OMP_NUM_THREADS=1 does
    not apply: the oracle is always given this count explicitly)."""
    try:
        return len(os.sched_getaffinity(0))
    except (AttributeError, OSError):
        return os.cpu_count() or 1


def env_int(name, default):
    try:
        return int(os.environ.get(name, default))
    except ValueError:
        return default


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return dict(hbm_gbs=p["hbm_gbs"], bf16=p["bf16_tflops"],
                    bf16_sustained=p.get("bf16_tflops_sustained", p["bf16_tflops"]),
                    source="measured")
    except (OSError, KeyError, ValueError):
        return dict(hbm_gbs=6650.0, bf16=1590.0, bf16_sustained=1400.0, source="fallback")


# ---------------------------------------------------------------- inputs

def gen_mixture_torch(n, d, clusters, seed, device):
    """Configs 0/1/3 on the device: centers ~U[0,100]^d, sigma 10, clipped to
    [0, 255], rounded; float32 (tests/data.py draws the same with NumPy)."""
    import torch

    g = torch.Generator(device=device)
    g.manual_seed(seed)
    centers = torch.rand((clusters, d), generator=g, device=device) * 100.0
    out = torch.empty((n, d), dtype=torch.float32, device=device)
    step = 1 << 20
    for i in range(0, n, step):
        m = min(step, n - i)
        lab = torch.randint(0, clusters, (m,), generator=g, device=device)
        x = centers[lab] + 10.0 * torch.randn((m, d), generator=g, device=device)
        out[i:i + m] = x.clamp_(0.0, 255.0).round_()
    return out


def gen_unit_torch(n, d, rank, seed, device):
    import torch

    g = torch.Generator(device=device)
    g.manual_seed(seed)
    basis = torch.randn((rank, d), generator=g, device=device)
    out = torch.empty((n, d), dtype=torch.float32, device=device)
    step = 1 << 18
    for i in range(0, n, step):
        m = min(step, n - i)
        x = torch.randn((m, d), generator=g, device=device) + \
            torch.randn((m, rank), generator=g, device=device) @ basis
        out[i:i + m] = x / x.norm(dim=1, keepdim=True)
    return out


def gen_codes_torch(n, nbytes, prototypes, flip, seed, device):
    """Config 4: random prototype codes XOR Bernoulli(flip) bits.  A noise
    byte b has probability flip^popc(b) (1-flip)^(8-popc(b)): one uniform per
    byte through that distribution's inverse CDF."""
    import torch

    g = torch.Generator(device=device)
    g.manual_seed(seed)
    protos = torch.randint(0, 256, (prototypes, nbytes), generator=g, device=device,
                           dtype=torch.int32).to(torch.uint8)
    pc = torch.tensor([bin(b).count("1") for b in range(256)], dtype=torch.float64)
    cdf = torch.cumsum(flip ** pc * (1.0 - flip) ** (8 - pc), 0)
    cdf = (cdf / cdf[-1]).to(torch.float32).to(device)
    out = torch.empty((n, nbytes), dtype=torch.uint8, device=device)
    step = 1 << 20
    for i in range(0, n, step):
        m = min(step, n - i)
        lab = torch.randint(0, prototypes, (m,), generator=g, device=device)
        u = torch.rand((m, nbytes), generator=g, device=device)
        noise = torch.searchsorted(cdf, u).clamp_(max=255).to(torch.uint8)
        out[i:i + m] = protos[lab] ^ noise
    return out


def make_inputs(w, device, seed=0):
    if w["kind"] == "allnn":
        base = gen_mixture_torch(w["n"], w["d"], w["clusters"], seed, device)
        return base, base
    if w["kind"] == "knn":
        base = gen_mixture_torch(w["n"], w["d"], w["clusters"], seed, device)
        q = gen_mixture_torch(w["nq"], w["d"], w["clusters"], seed + 1, device)
    elif w["kind"] == "knn-unit":
        base = gen_unit_torch(w["n"], w["d"], w["rank"], seed, device)
        q = gen_unit_torch(w["nq"], w["d"], w["rank"], seed + 1, device)
        if w.get("f16"):
            base = base.half().float()
            q = q.half().float()
    else:
        base = gen_codes_torch(w["n"], w["bytes"], w["prototypes"], w["flip"], seed, device)
        q = gen_codes_torch(w["nq"], w["bytes"], w["prototypes"], w["flip"], seed + 1, device)
    return base, q


# ---------------------------------------------------------------- clocks

class ClockSampler:
    """nvidia-smi samples of one GPU during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def start(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        time.sleep(0.3)

    def stop(self):
        if self.proc is None:
            return None
        time.sleep(0.2)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        with open(self.path) as f:
            for line in f:
                parts = [x.strip() for x in line.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    rows.append(dict(sm=float(parts[1]), max=float(parts[2]),
                                     power=float(parts[3]), active=parts[4],
                                     hw=parts[5], hw_thermal=parts[6], sw_thermal=parts[7],
                                     sw_power=parts[8]))
                except ValueError:
                    continue
        os.unlink(self.path)
        if not rows:
            return None
        max_power = max(r["power"] for r in rows)
        loaded = [r for r in rows if r["power"] >= 0.5 * max_power] or rows
        reasons = []
        for key, name in (("hw", "hw_slowdown"), ("hw_thermal", "hw_thermal_slowdown"),
                          ("sw_thermal", "sw_thermal_slowdown"), ("sw_power", "sw_power_cap")):
            if any(r[key].lower().startswith("active") for r in loaded):
                reasons.append(name)
        return {"sm_mhz": statistics.median(r["sm"] for r in loaded),
                "sm_max_mhz": max(r["max"] for r in rows), "reasons": reasons,
                "samples": len(loaded), "power_w_max": max_power}


def config_of(args, w, world):
    """The line's config, identical in both arms."""
    is_allnn = w["kind"] == "allnn"
    cfg = {"workload": args.workload, "desc": w["desc"], "n": w["n"], "queries": w["nq"],
           "k": w["k"],
           "parallelism": (f"rows to list split over {world} GPU(s), all rows on each"
                           if is_allnn else f"base rows sharded over {world} GPU(s)"),
           "l2_flush": f"{FLUSH_BYTES >> 20} MiB buffer written before every timed step "
                       f"(outside the per-step event spans)"}
    if getattr(args, "shard_of", 1) > 1:
        cfg["shard_of"] = args.shard_of
    if world > 1 and not is_allnn:
        cfg["exchange"] = ("peer memory over NVLink (PeerExchange)"
                           if getattr(args, "exchange", "peer") == "peer" and w["k"] <= 32
                           and world * w["k"] <= 768 and world <= 8 else "NCCL all-gather")
    if getattr(args, "entry", "default") == "noalloc":
        cfg["entry"] = "mlxvs_hamming_knn_noalloc (popcount kernel)"
    return cfg


# ---------------------------------------------------------------- CPU side

def cpu_sample_rate(w, base_np, q_np, budget_s, threads=0):
    """Oracle queries/s on a bounded sample of the workload (all base rows,
    a subset of the queries), calibrated to take about budget_s seconds."""
    from oracle import oracle as O

    def run(m):
        t = time.perf_counter()
        if w["kind"] == "hamming":
            O.hamming_knn(base_np, q_np[:m], w["k"], threads=threads)
        elif w["kind"] == "allnn":
            O.all_neighbors(base_np, w["k"], w["metric"], threads=threads, begin=0, end=m)
        else:
            O.brute_force_knn(base_np, q_np[:m], w["k"], w["metric"], threads=threads)
        return time.perf_counter() - t

    m = 8
    t = run(m)
    while t < 0.5 and m < q_np.shape[0]:
        m = min(q_np.shape[0], m * 4)
        t = run(m)
    rate = m / t
    m2 = int(min(q_np.shape[0], max(1, rate * budget_s)))
    t2 = run(m2) if m2 != m else t
    return m2 / t2, m2, t2


def reference_arm(args, w, peaks):
    """--impl reference: the CPU restatement of the reference's path (the
    reference itself needs macOS + Metal + MLX) on this host's cores."""
    rank = env_int("RANK", 0)
    if rank != 0:
        return 0
    import torch

    cores = host_threads()
    base, q = make_inputs(w, "cpu")
    base_np, q_np = base.numpy(), q.numpy()
    # each step: a bounded sample of the workload (all base rows, the first
    # m queries), m chosen so that the steps take about 90 s in all
    per_step = max(0.05, min(2.0, 90.0 / max(1, args.steps + args.warmup)))
    rate, m, _ = cpu_sample_rate(w, base_np, q_np, per_step, threads=cores)
    from oracle import oracle as O

    def step():
        if w["kind"] == "hamming":
            O.hamming_knn(base_np, q_np[:m], w["k"], threads=cores)
        elif w["kind"] == "allnn":
            O.all_neighbors(base_np, w["k"], w["metric"], threads=cores, begin=0, end=m)
        else:
            O.brute_force_knn(base_np, q_np[:m], w["k"], w["metric"], threads=cores)

    for _ in range(args.warmup):
        step()
    t = time.perf_counter()
    for _ in range(args.steps):
        step()
    el = time.perf_counter() - t
    value = m * args.steps / el
    sample = f"{m} of {w['nq']} queries against all {w['n']} base rows per step"
    if w["kind"] == "allnn":
        sample = (f"the lists of {m} of {w['n']} rows per step (a k + 1 search against all "
                  f"rows, then the row itself dropped)")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "queries/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": el / args.steps * 1e3, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": config_of(args, w, env_int("WORLD_SIZE", args.gpus)),
        "cpu_baseline": {"value": value, "unit": "queries/s", "cores": cores, "kind": "port",
                         "sample": sample, "threads": cores,
                         "omp_num_threads_env": os.environ.get("OMP_NUM_THREADS")},
        "e2e": {"value": value, "unit": "queries/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "note": "the reference (MLX + Metal, macOS only) cannot run here; its CPU "
                "restatement oracle/oracle.c (OpenMP, all cores) stands in",
    }
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------- parity

PARITY_SAMPLE = {"knn-unit": 200, "allnn": 2_000, "hamming": 500}


def check_parity(w, base, q, ids, dist, k, metric):
    """The last timed step's ids and distances against the oracle on every
    host thread.  Integer-valued L2 data (configs 0 and 1): every query,
    bit-exact.  Hamming: a sample of the queries, bit-exact.  all_neighbors:
    a sample of the rows to list, bit-exact.  Unit rows (config 2): a sample
    of the queries, distances within rtol = atol = 1e-4 of the oracle's and
    ids equal wherever the oracle's distances are not tied within that
    tolerance.  Returns counts of mismatching queries."""
    from oracle import oracle as O

    threads = host_threads()
    t0 = time.perf_counter()
    kind = w["kind"]
    nq = q.shape[0]
    m = nq if kind == "knn" else min(nq, PARITY_SAMPLE[kind])
    gi = ids[:m].cpu().numpy()
    gd = dist[:m].cpu().numpy()
    base_np = base.cpu().numpy()
    if kind == "allnn":
        oi, od = O.all_neighbors(base_np, k, metric, threads=threads, begin=0, end=m)
    elif kind == "hamming":
        oi, od = O.hamming_knn(base_np, q[:m].cpu().numpy(), k, threads=threads)
    else:
        oi, od = O.brute_force_knn(base_np, q[:m].cpu().numpy(), k, metric, threads=threads)
    if kind == "knn-unit":
        close = np.isclose(gd, od, rtol=1e-4, atol=1e-4)
        # a position may hold either of two rows whose scores tie within the
        # tolerance: compare ids only where the oracle's neighbours differ
        gap = np.abs(np.diff(od, axis=1)) > 1e-4 * np.maximum(1.0, np.abs(od[:, 1:]))
        sep = np.ones_like(od, dtype=bool)
        sep[:, 1:] &= gap
        sep[:, :-1] &= gap
        bad = ~close.all(axis=1) | ((gi != oi) & sep).any(axis=1)
        rule = "distances within rtol = atol = 1e-4, ids equal where not tied"
    else:
        bad = ~((gi == oi).all(axis=1) & (gd == od).all(axis=1))
        rule = "ids and distances bit-exact"
    what = "rows to list" if kind == "allnn" else "queries"
    return {"checked": int(m), "of": int(nq), "unit": what,
            "mismatched": int(bad.sum()), "rule": rule,
            "against": f"oracle/oracle.c on {threads} host threads",
            "seconds": round(time.perf_counter() - t0, 2)}


# ---------------------------------------------------------------- select arm

def select_arm(args, w, peaks):
    """topk_merge or refine on one GPU (rank 0 under torchrun): each step
    timed with CUDA events after an L2 flush, its HBM bytes against the
    measured copy bandwidth, and the first rows checked against the oracle."""
    if env_int("RANK", 0) != 0:
        return 0
    import torch

    import mlxvs_b200 as mv
    from oracle import oracle as O

    dev = torch.device("cuda", env_int("LOCAL_RANK", 0))
    torch.cuda.set_device(dev)
    g = torch.Generator(device=dev)
    g.manual_seed(0)
    k = w["k"]
    if w["kind"] == "topk":
        # integer-valued scores: many ties, which the reference's order breaks
        scores = (torch.randn((w["nq"], w["n"]), generator=g, device=dev) * 64.0).round_()

        def step():
            return mv.topk_merge(scores, None, None, 0, True, k)

        algo_bytes = scores.numel() * 4 + w["nq"] * k * 8
        kname = "topk_rows"
    else:
        base = gen_mixture_torch(w["n"], w["d"], w["clusters"], 0, dev)
        q = gen_mixture_torch(w["nq"], w["d"], w["clusters"], 1, dev)
        cand = torch.randint(0, w["n"], (w["nq"], w["c"]), generator=g, device=dev)

        def step():
            return mv.refine(base, q, cand, k, w["metric"])

        # every candidate row gathered once, its id, the queries
        algo_bytes = w["nq"] * w["c"] * (w["d"] * 4 + 8) + w["nq"] * w["d"] * 4
        kname = "refine"
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream(dev)
    flush = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device=dev)
    spans = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
             for _ in range(args.steps)]
    for i in range(args.steps):
        flush.fill_(i & 0x7F)
        spans[i][0].record(stream)
        out = step()
        spans[i][1].record(stream)
    torch.cuda.synchronize()
    ms = sum(a.elapsed_time(b) for a, b in spans) / args.steps
    m = 200
    ids = out[0][:m].cpu().numpy()
    vals = out[1][:m].cpu().numpy()
    if w["kind"] == "topk":
        oi, ov = O.topk_merge(scores[:m].cpu().numpy(), None, None, 0, True, k)
    else:
        oi, ov = O.refine(base.cpu().numpy(), q[:m].cpu().numpy(), cand[:m].cpu().numpy(), k,
                          w["metric"])
    mism = int(np.sum(np.any(ids != oi, axis=1) | np.any(vals != ov, axis=1)))
    gbs = algo_bytes / (ms / 1e3) / 1e9
    line = {
        "metric": f"{w['kind']} rows/s", "value": w["nq"] / (ms / 1e3), "unit": "rows/s",
        "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "dtype": "f32", "data": "synthetic (seeded)",
        "config": {"workload": args.workload, "desc": w["desc"],
                   "l2_flush": f"{FLUSH_BYTES >> 20} MiB buffer written before every step"},
        "roofline": {"bound": "hbm", "achieved": gbs, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": gbs / peaks["hbm_gbs"], "kernel": kname,
                     "algorithmic_per_step": f"{algo_bytes:.3e} bytes",
                     "peak_source": f"{peaks['source']} copy bandwidth"},
        "parity": {"checked": m, "of": w["nq"], "unit": "rows", "mismatched": mism,
                   "rule": "ids and scores bit-exact", "against": "oracle/oracle.py"},
    }
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------- GPU arm

def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--workload", default=DEFAULT_WORKLOAD, choices=sorted(WORKLOADS))
    ap.add_argument("--e2e-steps", type=int, default=5)
    ap.add_argument("--cpu-budget", type=float, default=12.0,
                    help="seconds of oracle work for cpu_baseline (rank 0, N=1)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-parity", action="store_true",
                    help="skip the post-timing comparison with the oracle")
    ap.add_argument("--entry", default="default", choices=["default", "noalloc"],
                    help="Hamming workloads at N=1: noalloc times mlxvs_hamming_knn_noalloc "
                         "(the popcount kernel, caller-owned outputs) instead of "
                         "mlxvs_hamming_knn_device")
    ap.add_argument("--exchange", default="peer", choices=["peer", "nccl"],
                    help="N > 1: the ranks' key lists merged from peer memory over NVLink "
                         "(PeerExchange) or through an NCCL all-gather")
    ap.add_argument("--shard-of", type=int, default=1,
                    help="one process searching the shard rank 0 holds at N GPUs (for "
                         "per-rank profiles on one GPU); the line is not a bench value")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    w = WORKLOADS[args.workload]
    peaks = load_peaks()
    if args.impl == "reference":
        return reference_arm(args, w, peaks)
    if w["kind"] in ("topk", "refine"):
        return select_arm(args, w, peaks)

    import torch
    import torch.distributed as dist

    import mlxvs_b200 as mv
    from mlxvs_b200 import distributed as mvd

    world = env_int("WORLD_SIZE", 1)
    rank = env_int("RANK", 0)
    local = env_int("LOCAL_RANK", 0)
    if world != args.gpus and world > 1:
        print(f"warning: WORLD_SIZE={world} but --gpus {args.gpus}", file=sys.stderr)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)

    def barrier():
        if world > 1:
            dist.barrier()

    # inputs: every rank draws the same seeded data and keeps its shard
    base, q = make_inputs(w, dev)
    bounds = mvd.shard_bounds(w["n"], world)
    lo, hi = bounds[rank], bounds[rank + 1]
    if world == 1 and args.shard_of > 1:
        # rank 0's shard (or share of the rows to list) at N = shard_of
        lo, hi = 0, mvd.shard_bounds(w["n"], args.shard_of)[1]
    is_allnn = w["kind"] == "allnn"
    # all_neighbors splits the rows to list (queries) over the GPUs, each
    # holding all rows; the others split the base rows
    shard = base if is_allnn else base[lo:hi].contiguous()
    full_base = base
    emulated = world == 1 and args.shard_of > 1
    k = w["k"]
    is_hamming = w["kind"] == "hamming"
    metric = None if is_hamming else w["metric"]
    stream = torch.cuda.current_stream(dev)
    noalloc_out = None
    if args.entry == "noalloc":
        if not is_hamming or world > 1:
            raise SystemExit("--entry noalloc is for Hamming workloads at N=1")
        noalloc_out = (torch.empty((w["nq"], k), dtype=torch.int32, device=dev),
                       torch.empty((w["nq"], k), dtype=torch.float32, device=dev))

    # N > 1: one exchange buffer per rank for every step's key lists
    exch = None
    if world > 1 and not is_allnn and args.exchange == "peer" and \
            world <= mvd.PeerExchange.MAX_WORLD and k <= 32 and world * k <= 768:
        exch = mvd.PeerExchange(w["nq"] * k)

    def step():
        if is_allnn:
            if world == 1 and not emulated:
                return mv.all_neighbors(shard, k, metric, algo="brute_force")
            return mv.all_neighbors_rows(shard, k, metric, begin=lo, end=hi)
        if world == 1:
            if is_hamming and noalloc_out is not None:
                return mv.hamming_knn_noalloc(shard, q, k, *noalloc_out)
            if is_hamming:
                return mv.hamming_knn(shard, q, k)
            return mv.brute_force_knn(shard, q, k, metric)
        if is_hamming:
            return mvd.sharded_hamming_knn(shard, q, k, id_offset=lo, exchange=exch)
        return mvd.sharded_brute_force_knn(shard, q, k, metric, id_offset=lo, exchange=exch)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    mv.synchronize()

    uuid = getattr(torch.cuda.get_device_properties(dev), "uuid", None)
    gpu_id = f"GPU-{uuid}" if uuid is not None else str(local)
    sampler = ClockSampler(gpu_id) if rank == 0 else None
    if sampler:
        sampler.start()
    # L2 (126 MB) is flushed before every timed step by writing a buffer of
    # twice its size: a rank's shard is smaller than L2 from N = 8 on (64 MB
    # of fp32 rows), so "inputs larger than L2" would not hold at every N.
    # Each step is timed alone with CUDA events on the launching stream, the
    # flushes between the spans; the step time is the sum of the spans.
    flush = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device=dev)
    spans = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
             for _ in range(args.steps)]
    barrier()
    torch.cuda.synchronize()
    for i in range(args.steps):
        flush.fill_(i & 0x7F)
        spans[i][0].record(stream)
        ids, dist_out = step()
        spans[i][1].record(stream)
    torch.cuda.synchronize()
    barrier()
    elapsed_ms = sum(a.elapsed_time(b) for a, b in spans)
    clocks = sampler.stop() if sampler else None
    # per-kernel times from CUDA events around each launch, in a separate
    # pass of the same steps (the events would otherwise add about 1 % to
    # the timed steps)
    prof_steps = min(args.steps, 20)
    mv.profile_enable(True)
    for i in range(prof_steps):
        flush.fill_(i & 0x7F)
        step()
    torch.cuda.synchronize()
    kname = "hamming_topk" if is_hamming else "gemm_topk"
    kern_ms, kern_launches = mv.profile_read(kname)
    if is_hamming and kern_launches == 0:  # the tensor-core path ran
        kname = "hamming_mma"
        kern_ms, kern_launches = mv.profile_read(kname)
    issued_ops = mv.profile_issued(kname)
    coll_ms, coll_launches = mv.profile_read("gemm_collect")
    if coll_launches > 0:
        issued_ops += mv.profile_issued("gemm_collect")
        # k > 32: a sampled pass (lists of 1/4 of the base) and a collecting
        # pass over the whole base make up one search; both are counted
        kname = "gemm_topk (sampled pass) + gemm_collect"
        kern_ms += coll_ms
        kern_launches = coll_launches
    # device time per step of each of the library's kernels (rank 0's
    # profiled pass); the rest of the step is the host's part and, for
    # N > 1, the all-gather
    step_breakdown = {}
    for name in ("prep", "gemm_topk", "gemm_topk_skipped", "gemm_collect", "hamming_mma",
                 "hamming_topk", "select_keys", "rescore", "merge", "fill"):
        ms, nl = mv.profile_read(name)
        if nl:
            step_breakdown[name] = ms / prof_steps
    _, all_launches = mv.profile_read(None)
    # launches of this library's kernels in the timed steps (the same per step)
    all_launches = all_launches * args.steps // max(prof_steps, 1)
    mv.profile_enable(False)
    mv.synchronize()
    if world > 1 and not is_allnn:
        # the sharded step in its parts, each bracketed by CUDA events on the
        # launching stream: this rank's search (prep, fused kernel, merge of
        # its units' lists), then either the peer exchange's merge (its wait
        # for every rank's keys included) or the NCCL all-gather of the
        # [nq, k] keys (which also waits for the slowest rank) and the merge
        kind = "hamming" if is_hamming else metric
        mq = q if metric == "l2" else None
        names = (("rank_search", "exchange_merge") if exch is not None else
                 ("rank_search", "all_gather", "final_merge"))
        parts = {n: 0.0 for n in names}
        for i in range(prof_steps):
            flush.fill_(i & 0x7F)
            ev = [torch.cuda.Event(enable_timing=True) for _ in range(len(names) + 1)]
            ev[0].record(stream)
            if exch is not None:
                if is_hamming:
                    exch.hamming_keys(shard, q, k, lo)
                    ev[1].record(stream)
                    exch.merge(q.shape[0], k, "hamming")
                else:
                    qf = exch.knn_keys(shard, q, k, metric, lo)
                    ev[1].record(stream)
                    exch.merge(q.shape[0], k, metric, qf)
                ev[2].record(stream)
            else:
                keys = (mv.hamming_keys(shard, q, k, id_offset=lo) if is_hamming else
                        mv.knn_keys(shard, q, k, metric, id_offset=lo))
                ev[1].record(stream)
                lists = mvd.gather_lists(keys)
                ev[2].record(stream)
                mv.merge_keys(lists, k, kind, mq)
                ev[3].record(stream)
            torch.cuda.synchronize()
            for j, name in enumerate(names):
                parts[name] += ev[j].elapsed_time(ev[j + 1]) / prof_steps
        step_breakdown.update(parts)
        # the slowest rank's fused kernel sets when the all-gather can finish
        t = torch.tensor([kern_ms / max(kern_launches, 1)], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        step_breakdown["kernel_max_over_ranks"] = float(t.item())
    if world > 1:
        t = torch.tensor([elapsed_ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        elapsed_ms = float(t.item())

    # parity of the last timed step's output with the oracle (rank 0, after
    # timing): every query for the integer-valued configs, a bounded sample
    # of the queries (or of the rows to list) for the others
    parity = None
    if rank == 0 and not args.no_parity and not emulated:
        parity = check_parity(w, full_base, q, ids, dist_out, k, metric)
    # e2e: the public API on host (pinned) buffers, copies inside the region
    # (every rank starts it together: rank 0 may have spent seconds on the
    # parity check, and a peer exchange waits for all ranks)
    barrier()
    e2e = None
    if args.e2e_steps > 0:
        base_h = shard.cpu().pin_memory()
        q_h = q.cpu().pin_memory()
        if world == 1:
            bnp, qnp = base_h.numpy(), q_h.numpy()

            def e2e_step():
                if is_allnn:
                    return mv.all_neighbors(bnp, k, metric, algo="brute_force")
                if is_hamming:
                    return mv.hamming_knn(bnp, qnp, k)
                return mv.brute_force_knn(bnp, qnp, k, metric)
        else:
            def e2e_step():
                sd = base_h.to(dev, non_blocking=True)
                if is_allnn:
                    i, d_ = mv.all_neighbors_rows(sd, k, metric, begin=lo, end=hi)
                    return i.cpu(), d_.cpu()
                qd = q_h.to(dev, non_blocking=True)
                if is_hamming:
                    i, d_ = mvd.sharded_hamming_knn(sd, qd, k, id_offset=lo, exchange=exch)
                else:
                    i, d_ = mvd.sharded_brute_force_knn(sd, qd, k, metric, id_offset=lo,
                                                        exchange=exch)
                return i.cpu(), d_.cpu()
        e2e_step()
        torch.cuda.synchronize()
        barrier()
        te = time.perf_counter()
        for _ in range(args.e2e_steps):
            e2e_step()
        torch.cuda.synchronize()
        e2e_s = time.perf_counter() - te
        barrier()
        if world > 1:
            t = torch.tensor([e2e_s], dtype=torch.float64, device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            e2e_s = float(t.item())
        h2d = shard.numel() * shard.element_size() + q.numel() * q.element_size()
        d2h = w["nq"] * k * 8
        if is_allnn:  # the rows are the queries; this rank's lists come back
            h2d = shard.numel() * shard.element_size()
            d2h = (hi - lo) * k * 8
        e2e = {"value": w["nq"] * args.e2e_steps / e2e_s, "unit": "queries/s",
               "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
               "steps": args.e2e_steps, "path": "mlxvs_brute_force_knn (C API, host buffers)"
               if world == 1 else "mlxvs_b200.distributed on pinned host buffers"}
        if is_allnn:
            e2e["path"] = ("mlxvs_all_neighbors (C API, host buffers)" if world == 1 else
                           "mlxvs_all_neighbors_device per rank on pinned host buffers")

    # roofline of the dominant kernel (rank 0's launches)
    roof = None
    step_s = elapsed_ms / args.steps / 1e3
    if kern_launches > 0:
        per_launch_s = kern_ms / kern_launches / 1e3
        n_local = hi - lo
        traffic, traffic_src = load_traffic(
            args.workload + ("+noalloc" if noalloc_out is not None else ""),
            args.shard_of if emulated else world)
        if is_hamming and kname == "hamming_mma":
            # codes as +-1 int8 on the tensor cores: 2 * Q * N * bits integer
            # ops per launch, against twice the measured bf16 rate (int8 runs
            # at twice the bf16 rate on this part; no int8 peak is measured)
            bits = w["bytes"] * 8
            ops = 2.0 * w["nq"] * n_local * bits
            ach = ops / per_launch_s / 1e12
            peak = 2.0 * peaks["bf16"]
            roof = {"bound": "tensor", "achieved": ach, "peak": peak, "unit": "TOPS (int8)",
                    "frac": ach / peak,
                    "frac_of_sustained": ach / (2.0 * peaks["bf16_sustained"]),
                    "step_frac": ops / step_s / 1e12 / peak,
                    "issued_frac": issued_ops / kern_launches / per_launch_s / 1e12 / peak,
                    "traffic": traffic, "traffic_source": traffic_src,
                    "peak_source": f"2 x {peaks['source']} bf16 burst",
                    "kernel": kname, "kernel_ms": per_launch_s * 1e3,
                    "algorithmic_per_launch": f"2*Q*N*bits = {ops:.3e} int8 ops "
                                              f"({w['nq'] * n_local * (bits // 32):.3e} "
                                              f"32-bit popcounts' worth)",
                    "issued_per_launch": f"{issued_ops / kern_launches:.3e} int8 ops (padded "
                                         f"query blocks x tiles x K)"}
        elif is_hamming:
            # the popcount kernel: 32-bit popcounts per launch, and the codes
            # it reads once per pass over the base against HBM bandwidth
            # POPC issues to the XU pipe: 16 lanes per clock per SM, taken
            # at the SM clock sampled during the timed steps
            words = w["bytes"] // 4
            pops = w["nq"] * n_local * words
            gbs = n_local * w["bytes"] / per_launch_s / 1e9
            sms = torch.cuda.get_device_properties(dev).multi_processor_count
            mhz = (clocks or {}).get("sm_mhz") or 1965.0
            xu_peak = 16.0 * sms * mhz * 1e6 / 1e12
            ach = pops / per_launch_s / 1e12
            roof = {"bound": "int-pipe (XU, POPC)", "achieved": ach,
                    "unit": "Tpopc32/s", "peak": xu_peak, "frac": ach / xu_peak,
                    "peak_source": f"16 POPC per clock per SM x {sms} SMs x {mhz:.0f} MHz "
                                   f"(sampled SM clock; the XU pipe's issue rate)",
                    "hbm_gbs_codes_once": gbs, "traffic": traffic,
                    "traffic_source": traffic_src,
                    "kernel": kname, "kernel_ms": per_launch_s * 1e3,
                    "algorithmic_per_launch": f"{pops:.3e} 32-bit popcounts"}
        else:
            flops = 2.0 * w["nq"] * n_local * w["d"]
            if is_allnn:  # this rank's rows against all rows
                flops = 2.0 * (hi - lo) * w["n"] * w["d"]
            ach = flops / per_launch_s / 1e12
            peak = peaks["bf16"]
            roof = {"bound": "tensor", "achieved": ach, "peak": peak, "unit": "TFLOP/s",
                    "frac": ach / peak,
                    "frac_of_sustained": ach / peaks["bf16_sustained"],
                    "step_frac": flops / step_s / 1e12 / peak,
                    "issued_frac": issued_ops / kern_launches / per_launch_s / 1e12 / peak,
                    "traffic": traffic, "traffic_source": traffic_src,
                    "peak_source": f"{peaks['source']} bf16 burst (dense cuBLAS GEMM)",
                    "kernel": kname, "kernel_ms": per_launch_s * 1e3,
                    "algorithmic_per_launch": f"2*Q*N*D = {flops:.3e} FLOP",
                    "issued_per_launch": f"{issued_ops / kern_launches:.3e} FLOP (padded query "
                                         f"blocks x tiles x (passes x padded D + 16 for "
                                         f"|b|^2), sampled pass included)"}
        roof["per_step_ms"] = step_breakdown
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        base_np = shard.cpu().numpy()
        q_np = q.cpu().numpy()
        threads = host_threads()
        rate, m, t = cpu_sample_rate(w, base_np, q_np, args.cpu_budget, threads=threads)
        what = (f"the lists of {m} rows (k + 1 search against all {w['n']} rows, then the "
                f"row itself dropped)" if is_allnn else
                f"{m} queries against all {w['n']} base rows")
        cpu = {"value": rate, "unit": "queries/s", "cores": threads, "kind": "port",
               "sample": f"{what} ({t:.1f} s, OpenMP on {threads} host threads)"}

    if rank == 0:
        value = w["nq"] * args.steps / (elapsed_ms / 1e3)
        line = {
            "metric": METRIC, "value": value, "unit": "queries/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": elapsed_ms / args.steps, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None,
            "dtype": ("s8" if kname == "hamming_mma" else "u8") if is_hamming else "f16",
            "data": "synthetic (seeded, BASELINE distributions)",
            "config": config_of(args, w, world),
            "roofline": roof, "cpu_baseline": cpu, "e2e": e2e,
            "gpu_launches": int(all_launches), "clocks": clocks,
            "parity": parity,
        }
        if emulated:
            line["note"] = (f"one GPU searching the shard rank 0 holds at N={args.shard_of} "
                            f"(rows {lo}..{hi}); a profiling aid, not a bench value")
        print(json.dumps(line), flush=True)
    if exch is not None:
        torch.cuda.synchronize()
        barrier()
        exch.close()
    if world > 1:
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
