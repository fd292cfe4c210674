"""mlxvs_b200: exact k-nearest-neighbor search on NVIDIA B200 (sm_100a).

A drop-in for mlxVS's exact k-NN entry points (python/mlxvs/__init__.py:106-115
of the reference):

    ids, distances = brute_force_knn(base, queries, k, metric="l2")
    ids, distances = hamming_knn(rows, queries, k)

NumPy arrays (or anything array-like) go through the C API's host-memory
entry points and come back as NumPy arrays; CUDA torch tensors stay on the
device and come back as torch tensors on the same device, computed on the
current torch stream (or `stream=`).

ids are int32 [nq, k], -1 where fewer than k rows exist; distances are
float32 [nq, k]: squared L2 ascending (+inf where missing), inner product or
cosine similarity descending (-inf where missing).  Ties keep the lower id.

Everything runs in libmlxvs_b200.so (hand-written sm_100a kernels); there is
no CPU fallback: without the library or a B200 the calls raise.
"""

import ctypes
import enum
import os

import numpy as np

__all__ = [
    "Metric",
    "GraphBuild",
    "brute_force_knn",
    "all_neighbors",
    "all_neighbors_rows",
    "topk_merge",
    "refine",
    "hamming_knn",
    "hamming_knn_noalloc",
    "knn_keys",
    "hamming_keys",
    "merge_keys",
    "library_path",
    "version",
]

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "libmlxvs_b200.so")
_lib = None


class Metric(enum.IntEnum):
    """How two rows compare (the reference's mlxvs.Metric, same values)."""

    inner_product = 0
    l2 = 1
    cosine = 2


KIND_HAMMING = 3


def library_path():
    return _LIB_PATH


def _load():
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(_LIB_PATH):
        raise RuntimeError(
            "mlxvs_b200: libmlxvs_b200.so is not built (python -m mlxvs_b200.build)")
    lib = ctypes.CDLL(_LIB_PATH)
    p, i64, i32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32
    sig = {
        "mlxvs_brute_force_knn": [p, i64, p, i64, i32, i32, ctypes.c_int, p, p],
        "mlxvs_hamming_knn": [p, i64, p, i64, i32, i32, p, p],
        "mlxvs_brute_force_knn_device": [p, i64, p, i64, i32, i32, ctypes.c_int, p, p, p],
        "mlxvs_hamming_knn_device": [p, i64, p, i64, i32, i32, p, p, p],
        "mlxvs_hamming_knn_noalloc": [p, i64, p, i64, i32, i32, p, p, p],
        "mlxvs_knn_keys_device": [p, i64, p, i64, i32, i32, ctypes.c_int, i64, p, p],
        "mlxvs_hamming_keys_device": [p, i64, p, i64, i32, i32, i64, p, p],
        "mlxvs_all_neighbors": [p, i64, i32, i32, ctypes.c_int, p, p],
        "mlxvs_topk_merge": [p, i64, i32, p, p, i32, i32, i32, p, p],
        "mlxvs_topk_merge_device": [p, i64, i32, p, p, i32, i32, i32, p, p, p],
        "mlxvs_refine": [p, i64, i32, p, i64, p, i32, i32, ctypes.c_int, p, p],
        "mlxvs_refine_device": [p, i64, i32, p, i64, p, i32, i32, ctypes.c_int, p, p, p],
        "mlxvs_all_neighbors_device": [p, i64, i32, i32, ctypes.c_int, i64, i64, p, p, p],
        "mlxvs_merge_keys_device": [p, i32, i64, i32, i32, p, i32, p, p, p],
        "mlxvs_exchange_create": [i32, i32, i64, ctypes.POINTER(ctypes.c_void_p)],
        "mlxvs_exchange_handle": [p, p],
        "mlxvs_exchange_open": [p, i32, p],
        "mlxvs_exchange_keys": [p, ctypes.c_uint32, ctypes.POINTER(ctypes.c_void_p)],
        "mlxvs_exchange_merge_device": [p, ctypes.c_uint32, i64, i32, i32, p, i32, p, p, p],
        "mlxvs_exchange_destroy": [p],
        "mlxvs_device_synchronize": [p],
        "mlxvs_profile_enable": [i32],
        "mlxvs_profile_read": [ctypes.c_char_p, ctypes.POINTER(ctypes.c_double),
                               ctypes.POINTER(ctypes.c_int64)],
        "mlxvs_profile_issued": [ctypes.c_char_p, ctypes.POINTER(ctypes.c_double)],
    }
    for name, args in sig.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = ctypes.c_int
    lib.mlxvs_last_error.restype = ctypes.c_char_p
    lib.mlxvs_last_error.argtypes = []
    lib.mlxvs_version.restype = ctypes.c_char_p
    lib.mlxvs_version.argtypes = []
    _lib = lib
    return lib


def version():
    return _load().mlxvs_version().decode()


def _check(rc):
    if rc == 0:
        return
    msg = _lib.mlxvs_last_error().decode()
    if rc == 1:
        raise ValueError(msg)
    raise RuntimeError(msg)


def _metric(metric):
    """A Metric from a Metric, its value or its name (python/mlxvs/__init__.py:80-103)."""
    if isinstance(metric, str):
        try:
            return Metric[metric]
        except KeyError:
            names = ", ".join(repr(n) for n in Metric.__members__)
            raise ValueError(f"unknown Metric {metric!r}; one of {names}") from None
    try:
        return Metric(int(metric))
    except (TypeError, ValueError):
        raise ValueError(f"unknown Metric {metric!r}") from None


def _is_torch(x):
    return type(x).__module__.startswith("torch") and hasattr(x, "is_cuda")


def _host_float_rows(x, op, name):
    """float_rows (src/utils.h:18-29) on host arrays: 2-D, real, as float32."""
    if _is_torch(x):
        x = x.detach().cpu().float().numpy() if x.dtype != _torch().bool else x.numpy()
    a = np.asarray(x)
    if a.ndim != 2:
        raise ValueError(f"[{op}] {name} must be 2-D [n, d].")
    if a.dtype == np.bool_ or np.iscomplexobj(a) or not np.issubdtype(a.dtype, np.number):
        raise ValueError(f"[{op}] {name} must be real numbers.")
    return np.ascontiguousarray(a, dtype=np.float32)


def _torch():
    import torch

    return torch


def _dev_float_rows(x, op, name):
    torch = _torch()
    if x.dim() != 2:
        raise ValueError(f"[{op}] {name} must be 2-D [n, d].")
    if x.dtype == torch.bool or x.is_complex():
        raise ValueError(f"[{op}] {name} must be real numbers.")
    return x.to(torch.float32).contiguous()


def _stream_handle(stream, device):
    if stream is None:
        return ctypes.c_void_p(_torch().cuda.current_stream(device).cuda_stream)
    if isinstance(stream, int):
        return ctypes.c_void_p(stream)
    return ctypes.c_void_p(stream.cuda_stream)


def brute_force_knn(base, queries, k, metric=Metric.l2, *, tile_rows=65536, stream=None):
    """Exact k-nearest neighbors of every query among the base rows.

    Same arguments and results as the reference's mlxvs.brute_force_knn
    (python/bindings.cpp:37-75).  tile_rows is accepted for compatibility;
    the kernels choose their own tiling.
    """
    op = "mlxvs::brute_force_knn"
    m = _metric(metric)
    lib = _load()
    k = int(k)
    if _is_torch(base) and _is_torch(queries) and base.is_cuda and queries.is_cuda:
        torch = _torch()
        b = _dev_float_rows(base, op, "base")
        q = _dev_float_rows(queries, op, "queries")
        if b.shape[1] != q.shape[1]:
            raise ValueError(f"[{op}] base and queries must have the same number of columns.")
        if b.device != q.device:
            raise ValueError(f"[{op}] base and queries must be on the same device.")
        nq = q.shape[0]
        ids = torch.empty((nq, max(k, 0)), dtype=torch.int32, device=q.device)
        dist = torch.empty((nq, max(k, 0)), dtype=torch.float32, device=q.device)
        with torch.cuda.device(q.device):
            _check(lib.mlxvs_brute_force_knn_device(
                b.data_ptr(), b.shape[0], q.data_ptr(), nq, b.shape[1], k, int(m),
                ids.data_ptr(), dist.data_ptr(), _stream_handle(stream, q.device)))
        return ids, dist
    b = _host_float_rows(base, op, "base")
    q = _host_float_rows(queries, op, "queries")
    if b.shape[1] != q.shape[1]:
        raise ValueError(f"[{op}] base and queries must have the same number of columns.")
    nq = q.shape[0]
    ids = np.empty((nq, max(k, 0)), np.int32)
    dist = np.empty((nq, max(k, 0)), np.float32)
    _check(lib.mlxvs_brute_force_knn(
        b.ctypes.data, b.shape[0], q.ctypes.data, nq, b.shape[1], k, int(m),
        ids.ctypes.data, dist.ctypes.data))
    return ids, dist


class GraphBuild(enum.IntEnum):
    """How all_neighbors builds each cluster's graph (include/mlxvs/mlxvs.h:
    143-149)."""

    brute_force = 0
    nn_descent = 1


def _graph_build(algo):
    if isinstance(algo, str):
        try:
            return GraphBuild[algo]
        except KeyError:
            names = ", ".join(repr(n) for n in GraphBuild.__members__)
            raise ValueError(f"unknown GraphBuild {algo!r}; one of {names}") from None
    return GraphBuild(int(algo))


def all_neighbors(rows, k, metric=Metric.l2, *, algo=GraphBuild.nn_descent, n_clusters=0,
                  overlap_factor=2, brute_force_below=4096, max_cluster_rows=0, verbose=False,
                  max_iterations=24, termination_threshold=1e-4, fp16=True, seed=42,
                  stream=None):
    """k-nearest-neighbor graph of the rows: every row's k nearest other rows,
    nearest first, with the ids and distances of brute_force_knn (-1 and
    +inf / -inf where fewer than k other rows exist).

    Same arguments, checks and results as the reference's all_neighbors
    (python/bindings.cpp:1183-1215, src/all_neighbors.cpp:265-300) on its
    exact path: one cluster (n_clusters 0 or 1) built by brute force, which
    the reference takes for algo brute_force and, with nn_descent, for
    n <= max(brute_force_below, k + 1).  The clustered and NN-Descent builds
    are not part of this library and raise NotImplementedError.  The
    NN-Descent tuning arguments are accepted and unused.
    """
    op = "mlxvs::all_neighbors"
    m = _metric(metric)
    g = _graph_build(algo)
    lib = _load()
    k = int(k)
    on_device = _is_torch(rows) and rows.is_cuda
    if on_device:
        x = _dev_float_rows(rows, op, "rows")
    else:
        x = _host_float_rows(rows, op, "rows")
    n, d = int(x.shape[0]), int(x.shape[1])
    max_k = 128 if g == GraphBuild.nn_descent else 255
    if k < 1 or k > max_k or n < 2 or d < 1:
        raise ValueError(f"[{op}] 1 <= k <= {max_k}, n >= 2 and d >= 1")
    if n_clusters < 0 or n_clusters > n or overlap_factor < 1 or (
            n_clusters > 1 and overlap_factor > n_clusters):
        raise ValueError(
            f"[{op}] 0 <= n_clusters <= n and 1 <= overlap_factor <= n_clusters")
    exact = n_clusters <= 1 and (
        g == GraphBuild.brute_force or n <= max(int(brute_force_below), k + 1))
    if not exact:
        raise NotImplementedError(
            f"[{op}] only the exact one-cluster build is implemented (algo='brute_force' "
            "with n_clusters 0 or 1, or n <= brute_force_below)")
    if on_device:
        torch = _torch()
        ids = torch.empty((n, k), dtype=torch.int32, device=x.device)
        dist = torch.empty((n, k), dtype=torch.float32, device=x.device)
        with torch.cuda.device(x.device):
            _check(lib.mlxvs_all_neighbors_device(
                x.data_ptr(), n, d, k, int(m), 0, n, ids.data_ptr(), dist.data_ptr(),
                _stream_handle(stream, x.device)))
        return ids, dist
    ids = np.empty((n, k), np.int32)
    dist = np.empty((n, k), np.float32)
    _check(lib.mlxvs_all_neighbors(x.ctypes.data, n, d, k, int(m), ids.ctypes.data,
                                   dist.ctypes.data))
    return ids, dist


def all_neighbors_rows(rows, k, metric=Metric.l2, *, begin, end, stream=None):
    """The exact all_neighbors lists of rows begin .. end - 1 only (CUDA
    tensors): how devices that each hold all rows split the graph."""
    op = "mlxvs::all_neighbors"
    m = _metric(metric)
    lib = _load()
    torch = _torch()
    x = _dev_float_rows(rows, op, "rows")
    n, d = int(x.shape[0]), int(x.shape[1])
    ids = torch.empty((max(0, end - begin), int(k)), dtype=torch.int32, device=x.device)
    dist = torch.empty((max(0, end - begin), int(k)), dtype=torch.float32, device=x.device)
    with torch.cuda.device(x.device):
        _check(lib.mlxvs_all_neighbors_device(
            x.data_ptr(), n, d, int(k), int(m), int(begin), int(end), ids.data_ptr(),
            dist.data_ptr(), _stream_handle(stream, x.device)))
    return ids, dist


def topk_merge(scores, ids, best, id_offset, first, k, *, stream=None):
    """One merge step of the exact search: the best k of each row of scores
    [nq, t] (ids id_offset + column) together with the running lists ids
    (int32) and best (float32) [nq, k], which are ignored when first is set.
    Returns (ids int32 [nq, k], scores float32 [nq, k]), best first (higher
    score, then lower id as unsigned), -1 / -inf padded.

    Same arguments, checks and results as the reference's topk_merge
    (include/mlxvs/mlxvs.h:898-905, src/knn.cpp:37-69).  NumPy in, NumPy
    out; CUDA tensors in, CUDA tensors out.
    """
    op = "mlxvs::topk_merge"
    lib = _load()
    k = int(k)
    first = bool(first)
    if _is_torch(scores) and scores.is_cuda:
        torch = _torch()
        if scores.dim() != 2 or scores.dtype != torch.float32:
            raise ValueError(f"[{op}] scores must be float32 [nq, t]")
        sc = scores.contiguous()
        nq, t = int(sc.shape[0]), int(sc.shape[1])
        if not first:
            pi = ids.to(device=sc.device, dtype=torch.int32).contiguous()
            pb = best.to(device=sc.device, dtype=torch.float32).contiguous()
            if tuple(pi.shape) != (nq, k) or tuple(pb.shape) != (nq, k):
                raise ValueError(f"[{op}] ids and best must be [nq, k]")
        out_ids = torch.empty((nq, max(k, 0)), dtype=torch.int32, device=sc.device)
        out_sc = torch.empty((nq, max(k, 0)), dtype=torch.float32, device=sc.device)
        with torch.cuda.device(sc.device):
            _check(lib.mlxvs_topk_merge_device(
                sc.data_ptr(), nq, t, None if first else pi.data_ptr(),
                None if first else pb.data_ptr(), int(id_offset), int(first), k,
                out_ids.data_ptr(), out_sc.data_ptr(), _stream_handle(stream, sc.device)))
        return out_ids, out_sc
    sc = scores.detach().cpu().numpy() if _is_torch(scores) else np.asarray(scores)
    if sc.ndim != 2 or sc.dtype != np.float32:
        raise ValueError(f"[{op}] scores must be float32 [nq, t]")
    sc = np.ascontiguousarray(sc)
    nq, t = sc.shape
    pi = pb = None
    if not first:
        pi = np.ascontiguousarray(np.asarray(ids), dtype=np.int32)
        pb = np.ascontiguousarray(np.asarray(best), dtype=np.float32)
        if pi.shape != (nq, k) or pb.shape != (nq, k):
            raise ValueError(f"[{op}] ids and best must be [nq, k]")
    out_ids = np.empty((nq, max(k, 0)), np.int32)
    out_sc = np.empty((nq, max(k, 0)), np.float32)
    _check(lib.mlxvs_topk_merge(
        sc.ctypes.data, nq, t, None if first else pi.ctypes.data,
        None if first else pb.ctypes.data, int(id_offset), int(first), k,
        out_ids.ctypes.data, out_sc.ctypes.data))
    return out_ids, out_sc


def refine(dataset, queries, candidates, k, metric="l2", *, stream=None):
    """Exact re-ranking, as cuVS's refine: the k nearest of each query's
    candidate ids [nq, c] (ids outside [0, n) skipped) by exact distances,
    nearest first; (ids int32 [nq, k], distances float32 [nq, k]) as
    brute_force_knn returns them.  Equal distances keep the candidates'
    order; repeated candidates are all kept, as in the reference.

    Same arguments and results as the reference's refine
    (python/mlxvs/_ivf.py:158-185, src/ivf.cpp:1642-1708).  With NumPy
    inputs only the distinct candidate rows are copied to the device; with
    CUDA tensors everything stays on the device.
    """
    op = "mlxvs::refine"
    m = _metric(metric)
    lib = _load()
    k = int(k)
    if _is_torch(dataset) and dataset.is_cuda:
        torch = _torch()
        ds = _dev_float_rows(dataset, op, "dataset")
        q = queries if _is_torch(queries) else torch.as_tensor(np.asarray(queries))
        q = q.to(ds.device)
        if q.dim() == 1:
            q = q[None]
        q = _dev_float_rows(q, op, "queries")
        cand = candidates if _is_torch(candidates) else torch.as_tensor(np.asarray(candidates))
        cand = cand.to(device=ds.device, dtype=torch.int64)
        cand = torch.where((cand >= 0) & (cand < ds.shape[0]), cand, -1)
        cand = cand.to(torch.int32).contiguous()
        nq, d = int(q.shape[0]), int(q.shape[1])
        if ds.shape[1] != d or cand.dim() != 2 or cand.shape[0] != nq:
            raise ValueError(f"[{op}] dataset [n, d], queries [nq, d] and candidates [nq, c] "
                             "must match.")
        c = int(cand.shape[1])
        ids = torch.empty((nq, max(k, 0)), dtype=torch.int32, device=ds.device)
        dist = torch.empty((nq, max(k, 0)), dtype=torch.float32, device=ds.device)
        with torch.cuda.device(ds.device):
            _check(lib.mlxvs_refine_device(
                ds.data_ptr(), int(ds.shape[0]), d, q.data_ptr(), nq, cand.data_ptr(), c, k,
                int(m), ids.data_ptr(), dist.data_ptr(), _stream_handle(stream, ds.device)))
        return ids, dist
    ds = _host_float_rows(dataset, op, "dataset")
    q = np.asarray(queries.detach().cpu() if _is_torch(queries) else queries)
    if q.ndim == 1:
        q = q[None]
    q = _host_float_rows(q, op, "queries")
    cand = np.asarray(candidates.detach().cpu() if _is_torch(candidates) else candidates)
    nq, d = q.shape
    if ds.shape[1] != d or cand.ndim != 2 or cand.shape[0] != nq:
        raise ValueError(f"[{op}] dataset [n, d], queries [nq, d] and candidates [nq, c] "
                         "must match.")
    cand64 = cand.astype(np.int64)
    # ids outside the dataset (also those beyond int32) are skipped as -1
    cand32 = np.where((cand64 >= 0) & (cand64 < ds.shape[0]), cand64, -1).astype(np.int32)
    cand32 = np.ascontiguousarray(cand32)
    c = cand32.shape[1]
    ids = np.empty((nq, max(k, 0)), np.int32)
    dist = np.empty((nq, max(k, 0)), np.float32)
    _check(lib.mlxvs_refine(ds.ctypes.data, ds.shape[0], d, q.ctypes.data, nq, cand32.ctypes.data,
                            c, k, int(m), ids.ctypes.data, dist.ctypes.data))
    return ids, dist


def _host_codes(x, op, name):
    if _is_torch(x):
        x = x.detach().cpu().numpy()
    a = np.asarray(x)
    if a.ndim != 2 or a.dtype != np.uint8:
        raise ValueError(f"[{op}] {name} must be bit-packed uint8 [n, bytes].")
    return np.ascontiguousarray(a)


def hamming_knn(rows, queries, k, *, stream=None):
    """Exact k-NN by Hamming distance of bit-packed uint8 rows.

    Same arguments and results as the reference's mlxvs.hamming_knn
    (python/bindings.cpp:681-710): ids int32 [nq, k] and the Hamming
    distances as float32 [nq, k], nearest first, ties to the lower id.
    """
    op = "mlxvs::hamming_knn"
    lib = _load()
    k = int(k)
    if _is_torch(rows) and _is_torch(queries) and rows.is_cuda and queries.is_cuda:
        torch = _torch()
        for t, nm in ((rows, "rows"), (queries, "queries")):
            if t.dim() != 2 or t.dtype != torch.uint8:
                raise ValueError(f"[{op}] {nm} must be bit-packed uint8 [n, bytes].")
        if rows.shape[1] != queries.shape[1]:
            raise ValueError(f"[{op}] queries must have the rows' bytes.")
        r = rows.contiguous()
        q = queries.contiguous()
        nq = q.shape[0]
        ids = torch.empty((nq, max(k, 0)), dtype=torch.int32, device=q.device)
        dist = torch.empty((nq, max(k, 0)), dtype=torch.float32, device=q.device)
        with torch.cuda.device(q.device):
            _check(lib.mlxvs_hamming_knn_device(
                r.data_ptr(), r.shape[0], q.data_ptr(), nq, r.shape[1], k,
                ids.data_ptr(), dist.data_ptr(), _stream_handle(stream, q.device)))
        return ids, dist
    r = _host_codes(rows, op, "rows")
    q = _host_codes(queries, op, "queries")
    if r.shape[1] != q.shape[1]:
        raise ValueError(f"[{op}] queries must have the rows' bytes.")
    nq = q.shape[0]
    ids = np.empty((nq, max(k, 0)), np.int32)
    dist = np.empty((nq, max(k, 0)), np.float32)
    _check(lib.mlxvs_hamming_knn(
        r.ctypes.data, r.shape[0], q.ctypes.data, nq, r.shape[1], k,
        ids.ctypes.data, dist.ctypes.data))
    return ids, dist


def hamming_knn_noalloc(rows, queries, k, ids, dist, *, stream=None):
    """hamming_knn into caller-owned outputs, with no device allocation
    (mlxvs_hamming_knn_noalloc): rows and queries are uint8 CUDA tensors,
    ids int32 and dist float32 CUDA tensors of shape [nq, k].  Its scratch is
    one static array per GPU, so calls must not overlap and
    nq * (k + 1) * 8 bytes must fit in 16 MiB."""
    op = "mlxvs::hamming_knn"
    lib = _load()
    torch = _torch()
    for t, nm in ((rows, "rows"), (queries, "queries")):
        if not (_is_torch(t) and t.is_cuda and t.dim() == 2 and t.dtype == torch.uint8
                and t.is_contiguous()):
            raise ValueError(f"[{op}] {nm} must be bit-packed uint8 [n, bytes] on a CUDA "
                             "device, contiguous.")
    nq, k = queries.shape[0], int(k)
    for t, dt, nm in ((ids, torch.int32, "ids"), (dist, torch.float32, "dist")):
        if not (_is_torch(t) and t.is_cuda and t.dtype == dt and tuple(t.shape) == (nq, k)
                and t.is_contiguous()):
            raise ValueError(f"[{op}] {nm} must be a contiguous CUDA tensor [nq, k] of {dt}.")
    with torch.cuda.device(queries.device):
        _check(lib.mlxvs_hamming_knn_noalloc(
            rows.data_ptr(), rows.shape[0], queries.data_ptr(), nq, rows.shape[1], k,
            ids.data_ptr(), dist.data_ptr(), _stream_handle(stream, queries.device)))
    return ids, dist


def knn_keys(base, queries, k, metric=Metric.l2, *, id_offset=0, stream=None):
    """One shard's k best candidates per query as int64 keys [nq, k] (CUDA tensors).

    A key holds (order_bits(score) << 32) | ~id as a 64-bit pattern (see
    include/mlxvs_c.h); larger is better, 0 is an empty slot.
    """
    op = "mlxvs::brute_force_knn"
    torch = _torch()
    lib = _load()
    m = _metric(metric)
    b = _dev_float_rows(base, op, "base")
    q = _dev_float_rows(queries, op, "queries")
    if b.shape[1] != q.shape[1]:
        raise ValueError(f"[{op}] base and queries must have the same number of columns.")
    keys = torch.empty((q.shape[0], k), dtype=torch.int64, device=q.device)
    with torch.cuda.device(q.device):
        _check(lib.mlxvs_knn_keys_device(
            b.data_ptr(), b.shape[0], q.data_ptr(), q.shape[0], b.shape[1], int(k), int(m),
            int(id_offset), keys.data_ptr(), _stream_handle(stream, q.device)))
    return keys


def hamming_keys(rows, queries, k, *, id_offset=0, stream=None):
    """One shard's Hamming candidates as int64 keys [nq, k] (CUDA tensors)."""
    torch = _torch()
    lib = _load()
    r = rows.contiguous()
    q = queries.contiguous()
    if r.dtype != torch.uint8 or q.dtype != torch.uint8 or r.dim() != 2 or q.dim() != 2:
        raise ValueError("[mlxvs::hamming_knn] rows must be bit-packed uint8 [n, bytes].")
    if r.shape[1] != q.shape[1]:
        raise ValueError("[mlxvs::hamming_knn] queries must have the rows' bytes.")
    keys = torch.empty((q.shape[0], k), dtype=torch.int64, device=q.device)
    with torch.cuda.device(q.device):
        _check(lib.mlxvs_hamming_keys_device(
            r.data_ptr(), r.shape[0], q.data_ptr(), q.shape[0], r.shape[1], int(k),
            int(id_offset), keys.data_ptr(), _stream_handle(stream, q.device)))
    return keys


def merge_keys(lists, k, kind, queries=None, *, stream=None):
    """Best k of key lists [L, nq, k] (a CUDA int64 tensor) as (ids, distances).

    kind: a Metric (or its name) or "hamming".  L2 distances need the queries.
    """
    torch = _torch()
    lib = _load()
    kind = KIND_HAMMING if kind == "hamming" else int(_metric(kind))
    lists = lists.contiguous()
    L, nq, kk = lists.shape
    if kk != k:
        raise ValueError("[mlxvs::merge_keys] lists must be [L, nq, k].")
    ids = torch.empty((nq, k), dtype=torch.int32, device=lists.device)
    dist = torch.empty((nq, k), dtype=torch.float32, device=lists.device)
    qp, d = 0, 0
    if queries is not None:
        q = queries.to(torch.float32).contiguous()
        qp, d = q.data_ptr(), q.shape[1]
    with torch.cuda.device(lists.device):
        _check(lib.mlxvs_merge_keys_device(
            lists.data_ptr(), L, nq, int(k), kind, qp, d, ids.data_ptr(), dist.data_ptr(),
            _stream_handle(stream, lists.device)))
    return ids, dist


def synchronize(stream=None, device=None):
    """Waits for the stream and raises if a kernel recorded an error."""
    torch = _torch()
    dev = device if device is not None else torch.cuda.current_device()
    with torch.cuda.device(dev):
        _check(_load().mlxvs_device_synchronize(_stream_handle(stream, dev)))


def profile_enable(on=True):
    """Brackets every kernel launch with CUDA events (benchmarks); clears records."""
    _check(_load().mlxvs_profile_enable(1 if on else 0))


def profile_read(kernel=None):
    """(total device ms, launches) of the recorded launches of one kernel, or all."""
    ms = ctypes.c_double(0.0)
    n = ctypes.c_int64(0)
    name = kernel.encode() if kernel else None
    _check(_load().mlxvs_profile_read(name, ctypes.byref(ms), ctypes.byref(n)))
    return ms.value, n.value


def profile_issued(kernel=None):
    """Tensor-core operations (multiply-adds count 2) the recorded launches of
    one kernel, or of all, issued: padded query blocks x tiles x issued K."""
    ops = ctypes.c_double(0.0)
    name = kernel.encode() if kernel else None
    _check(_load().mlxvs_profile_issued(name, ctypes.byref(ops)))
    return ops.value
