"""Row-sharded exact k-NN across the GPUs of one node.

One process per GPU (torch.distributed, NCCL).  The base rows are split into
contiguous shards; every rank searches its shard for all queries with the
fused kernel, ids offset by the shard's first row (mlxvs_knn_keys_device),
so that each rank holds its k best candidates per query as 64-bit keys.
One all-gather of the [nq, k] keys (8 * nq * k bytes per rank) over NVLink
is the only exchange; the merge kernel then keeps the k best of the
world * k candidates per query (ties to the lower id, the reference's order)
and converts them to distances.  Lower ranks hold lower ids, so the result
equals the single-GPU search bit for bit.

This replaces the reference's single-device tile loop (src/knn.cpp:104-121,
merges at :117) with a cross-device one; the reference has no multi-GPU
path.
"""

import contextlib

import torch
import torch.distributed as dist

from . import (KIND_HAMMING, Metric, _metric, all_neighbors_rows, hamming_keys, knn_keys,
               merge_keys)

__all__ = ["shard_bounds", "gather_lists", "sharded_brute_force_knn", "sharded_hamming_knn",
           "sharded_all_neighbors"]


def shard_bounds(n, world):
    """Row ranges [b[r], b[r+1]) of the world's shards: contiguous, in rank order."""
    return [(r * n) // world for r in range(world + 1)]


def gather_lists(keys, group=None):
    """All ranks' [nq, k] key lists as one [world, nq, k] tensor (rank order)."""
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    if world == 1:
        return keys.unsqueeze(0)
    keys = keys.contiguous()
    if keys.is_cuda:
        out = torch.empty((world,) + tuple(keys.shape), dtype=keys.dtype, device=keys.device)
        dist.all_gather_into_tensor(out, keys, group=group)
        return out
    parts = [torch.empty_like(keys) for _ in range(world)]
    dist.all_gather(parts, keys, group=group)
    return torch.stack(parts)


def _on_stream(stream, device):
    """Makes `stream` torch's current stream for the block (nothing when it is
    None).  The search, the NCCL all-gather (which torch queues on its current
    stream) and every tensor allocated in between then share one stream, so
    the gather cannot read keys the search has not written yet.  A raw
    cudaStream_t handle (an int) is wrapped as an external stream."""
    if stream is None:
        return contextlib.nullcontext()
    if isinstance(stream, int):
        stream = torch.cuda.ExternalStream(stream, device=device)
    return torch.cuda.stream(stream)


def sharded_brute_force_knn(base_shard, queries, k, metric=Metric.l2, *, id_offset, group=None,
                            stream=None):
    """Exact k-NN of queries against the union of every rank's base shard.

    base_shard and queries are CUDA tensors (queries identical on every
    rank); id_offset is the global id of this shard's first row.  All work,
    the all-gather included, is queued on `stream` (default: torch's current
    stream).  Returns (ids int32 [nq, k], distances float32 [nq, k]) on every
    rank.
    """
    m = _metric(metric)
    with _on_stream(stream, queries.device):
        keys = knn_keys(base_shard, queries, k, m, id_offset=id_offset)
        lists = gather_lists(keys, group)
        return merge_keys(lists, k, m, queries if m == Metric.l2 else None)


def sharded_hamming_knn(rows_shard, queries, k, *, id_offset, group=None, stream=None):
    """Hamming version of sharded_brute_force_knn (uint8 codes)."""
    with _on_stream(stream, queries.device):
        keys = hamming_keys(rows_shard, queries, k, id_offset=id_offset)
        lists = gather_lists(keys, group)
        return merge_keys(lists, k, "hamming")


def sharded_all_neighbors(rows, k, metric=Metric.l2, *, group=None, stream=None, gather=True):
    """Exact k-NN graph of rows (a CUDA tensor, the same on every rank): each
    rank lists its contiguous share of the rows against all rows, with no
    exchange.  Returns (ids, distances) of the whole graph on every rank
    (gather: an all-gather of the lists), else this rank's [hi - lo, k]
    share and its (lo, hi)."""
    with _on_stream(stream, rows.device):
        return _sharded_all_neighbors(rows, k, metric, group, gather)


def _sharded_all_neighbors(rows, k, metric, group, gather):
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    rank = dist.get_rank(group) if dist.is_initialized() else 0
    n = rows.shape[0]
    b = shard_bounds(n, world)
    lo, hi = b[rank], b[rank + 1]
    ids, dst = all_neighbors_rows(rows, k, metric, begin=lo, end=hi)
    if not gather:
        return ids, dst, (lo, hi)
    if world == 1:
        return ids, dst
    # equal-sized pieces for the all-gather: pad to the largest share
    rows_max = max(b[r + 1] - b[r] for r in range(world))
    pad = rows_max - (hi - lo)
    if pad:
        ids = torch.cat([ids, ids.new_full((pad, k), -1)])
        dst = torch.cat([dst, dst.new_zeros((pad, k))])
    all_ids = torch.empty((world * rows_max, k), dtype=ids.dtype, device=ids.device)
    all_dst = torch.empty((world * rows_max, k), dtype=dst.dtype, device=dst.device)
    dist.all_gather_into_tensor(all_ids, ids.contiguous(), group=group)
    dist.all_gather_into_tensor(all_dst, dst.contiguous(), group=group)
    keep = torch.cat([torch.arange(r * rows_max, r * rows_max + b[r + 1] - b[r],
                                   device=ids.device) for r in range(world)])
    return all_ids[keep], all_dst[keep]


KIND = {"hamming": KIND_HAMMING}
