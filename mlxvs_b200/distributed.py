"""Row-sharded exact k-NN across the GPUs of one node.

One process per GPU (torch.distributed for set-up).  The base rows are split
into contiguous shards; every rank searches its shard for all queries with
the fused kernel, ids offset by the shard's first row (mlxvs_knn_keys_device),
so that each rank holds its k best candidates per query as 64-bit keys.
The ranks' [nq, k] key lists (8 * nq * k bytes each) are the only exchange:
with a PeerExchange every rank writes them into a buffer the others have
mapped (CUDA IPC) and one merge kernel reads all of them over NVLink, after
a one-warp kernel that publishes this rank's step and waits for the
others'; without one, an NCCL all-gather followed by the merge kernel.  The
merge keeps the k best of the world * k candidates per query (ties to the
lower id, the reference's order) and converts them to distances.  Lower
ranks hold lower ids, so the result equals the single-GPU search bit for
bit.

This replaces the reference's single-device tile loop (src/knn.cpp:104-121,
merges at :117) with a cross-device one; the reference has no multi-GPU
path.
"""

import contextlib
import ctypes

import torch
import torch.distributed as dist

from . import (KIND_HAMMING, Metric, _check, _dev_float_rows, _load, _metric, _stream_handle,
               all_neighbors_rows, hamming_keys, knn_keys, merge_keys)

__all__ = ["shard_bounds", "gather_lists", "PeerExchange", "sharded_brute_force_knn",
           "sharded_hamming_knn", "sharded_all_neighbors"]


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


class PeerExchange:
    """The ranks' key lists exchanged over NVLink instead of an NCCL
    all-gather (mlxvs_exchange_*): every rank writes its [nq, k] keys of a
    step into its own buffer and the merge kernel reads the peers' buffers
    directly (CUDA IPC mappings), after a kernel that publishes this rank's
    step and waits (bounded) for every other rank's.  One per process and
    device, created on every rank of the group at the same time (it
    exchanges the buffers' IPC handles with one all-gather); every rank must
    then run the same sequence of searches through it.  Needs k <= 32,
    world * k <= 768, world <= 8 and nq * k <= capacity_keys.
    """

    MAX_WORLD = 8

    def __init__(self, capacity_keys, group=None, device=None):
        self.lib = _load()
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None \
            else torch.device(device)
        self.capacity = int(capacity_keys)
        self.epoch = 0
        self.handle = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            _check(self.lib.mlxvs_exchange_create(self.world, self.rank, self.capacity,
                                                  ctypes.byref(self.handle)))
            mine = (ctypes.c_uint8 * 64)()
            _check(self.lib.mlxvs_exchange_handle(self.handle, mine))
            if self.world > 1:
                backend = dist.get_backend(group)
                where = self.device if backend == "nccl" else torch.device("cpu")
                t = torch.tensor(list(bytes(mine)), dtype=torch.uint8, device=where)
                parts = [torch.empty_like(t) for _ in range(self.world)]
                dist.all_gather(parts, t, group=group)
                for r, part in enumerate(parts):
                    h = (ctypes.c_uint8 * 64)(*part.cpu().tolist())
                    _check(self.lib.mlxvs_exchange_open(self.handle, r, h))
                dist.barrier(group=group)

    def fits(self, nq, k):
        return (self.handle.value is not None and 1 <= k <= 32 and self.world * k <= 768
                and nq * k <= self.capacity)

    def _next_slot(self):
        self.epoch += 1
        ptr = ctypes.c_void_p()
        _check(self.lib.mlxvs_exchange_keys(self.handle, self.epoch, ctypes.byref(ptr)))
        return ptr.value

    def _merge(self, nq, k, kind, queries, stream):
        ids = torch.empty((nq, k), dtype=torch.int32, device=self.device)
        dst = torch.empty((nq, k), dtype=torch.float32, device=self.device)
        qp, d = 0, 0
        if queries is not None:
            qp, d = queries.data_ptr(), queries.shape[1]
        _check(self.lib.mlxvs_exchange_merge_device(
            self.handle, self.epoch, nq, int(k), kind, qp, d, ids.data_ptr(), dst.data_ptr(),
            _stream_handle(stream, self.device)))
        return ids, dst

    def knn_keys(self, base_shard, queries, k, metric, id_offset, stream=None):
        """Step 1 of a search: this rank's k best keys of its shard, written
        into its slot of the next epoch.  Returns the float32 queries that
        step 2 (merge) takes for L2 distances."""
        op = "mlxvs::brute_force_knn"
        m = _metric(metric)
        b = _dev_float_rows(base_shard, op, "base")
        q = _dev_float_rows(queries, op, "queries")
        if b.shape[1] != q.shape[1]:
            raise ValueError(f"[{op}] base and queries must have the same number of columns.")
        with torch.cuda.device(self.device):
            slot = self._next_slot()
            _check(self.lib.mlxvs_knn_keys_device(
                b.data_ptr(), b.shape[0], q.data_ptr(), q.shape[0], b.shape[1], int(k), int(m),
                int(id_offset), slot, _stream_handle(stream, self.device)))
        return q

    def hamming_keys(self, rows_shard, queries, k, id_offset, stream=None):
        """knn_keys for bit-packed uint8 codes."""
        r = rows_shard.contiguous()
        q = queries.contiguous()
        if r.dtype != torch.uint8 or q.dtype != torch.uint8 or r.dim() != 2 or q.dim() != 2:
            raise ValueError("[mlxvs::hamming_knn] rows must be bit-packed uint8 [n, bytes].")
        if r.shape[1] != q.shape[1]:
            raise ValueError("[mlxvs::hamming_knn] queries must have the rows' bytes.")
        with torch.cuda.device(self.device):
            slot = self._next_slot()
            _check(self.lib.mlxvs_hamming_keys_device(
                r.data_ptr(), r.shape[0], q.data_ptr(), q.shape[0], r.shape[1], int(k),
                int(id_offset), slot, _stream_handle(stream, self.device)))

    def merge(self, nq, k, kind, queries=None, stream=None):
        """Step 2: publish this rank's keys of the epoch, wait for every
        rank's, merge them into (ids, distances); kind a Metric or "hamming"
        (L2 needs the float32 queries)."""
        kind = KIND_HAMMING if kind == "hamming" else int(_metric(kind))
        with torch.cuda.device(self.device):
            return self._merge(nq, k, kind, queries if kind == int(Metric.l2) else None, stream)

    def knn(self, base_shard, queries, k, metric, id_offset, stream=None):
        """This rank's search of its shard, then the exchange and merge."""
        q = self.knn_keys(base_shard, queries, k, metric, id_offset, stream)
        return self.merge(q.shape[0], k, metric, q, stream)

    def hamming(self, rows_shard, queries, k, id_offset, stream=None):
        self.hamming_keys(rows_shard, queries, k, id_offset, stream)
        return self.merge(queries.shape[0], k, "hamming", None, stream)

    def close(self):
        if self.handle.value is not None:
            with torch.cuda.device(self.device):
                self.lib.mlxvs_exchange_destroy(self.handle)
            self.handle = ctypes.c_void_p()


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
                            stream=None, exchange=None):
    """Exact k-NN of queries against the union of every rank's base shard.

    base_shard and queries are CUDA tensors (queries identical on every
    rank); id_offset is the global id of this shard's first row.  All work,
    the exchange included, is queued on `stream` (default: torch's current
    stream).  With a PeerExchange (that fits nq and k) the ranks' lists are
    merged straight from the peers' memory; otherwise through an NCCL
    all-gather.  Returns (ids int32 [nq, k], distances float32 [nq, k]) on
    every rank.
    """
    m = _metric(metric)
    if exchange is not None and exchange.fits(queries.shape[0], k):
        with _on_stream(stream, queries.device):
            return exchange.knn(base_shard, queries, k, m, id_offset)
    with _on_stream(stream, queries.device):
        keys = knn_keys(base_shard, queries, k, m, id_offset=id_offset)
        lists = gather_lists(keys, group)
        return merge_keys(lists, k, m, queries if m == Metric.l2 else None)


def sharded_hamming_knn(rows_shard, queries, k, *, id_offset, group=None, stream=None,
                        exchange=None):
    """Hamming version of sharded_brute_force_knn (uint8 codes)."""
    if exchange is not None and exchange.fits(queries.shape[0], k):
        with _on_stream(stream, queries.device):
            return exchange.hamming(rows_shard, queries, k, id_offset)
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
