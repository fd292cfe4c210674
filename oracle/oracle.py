"""ctypes front end of the CPU oracle (oracle.c).

TEST INFRASTRUCTURE ONLY: tests/, __graft_entry__.smoke() and bench.py's
cpu_baseline / reference leg use it as the checker or the CPU baseline.
Nothing in the mlxvs_b200 package imports this module.

The functions mirror the reference's Python API shape
(python/mlxvs/__init__.py:106-115): numpy in, (ids int32 [nq,k],
distances float32 [nq,k]) out.
"""

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")
_lib = None

IP, L2, COSINE = 0, 1, 2
_METRICS = {"inner_product": IP, "l2": L2, "cosine": COSINE}


def build():
    """Compiles liboracle.so with the committed Makefile."""
    env = dict(os.environ)
    subprocess.run(["make", "-s", "-C", _HERE], check=True, env=env)


def _load():
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(_LIB_PATH):
        build()
    lib = ctypes.CDLL(_LIB_PATH)
    i64, i32, p = ctypes.c_int64, ctypes.c_int32, ctypes.c_void_p
    lib.oracle_brute_force_knn.argtypes = [p, i64, p, i64, i32, i32, i32, p, p, i32]
    lib.oracle_brute_force_knn.restype = ctypes.c_int
    lib.oracle_hamming_knn.argtypes = [p, i64, p, i64, i32, i32, p, p, i32]
    lib.oracle_hamming_knn.restype = ctypes.c_int
    lib.oracle_knn_keys.argtypes = [p, i64, p, i64, i32, i32, i32, i64, p, i32]
    lib.oracle_knn_keys.restype = ctypes.c_int
    lib.oracle_merge_keys.argtypes = [p, i32, i64, i32, p]
    lib.oracle_merge_keys.restype = None
    lib.oracle_key.argtypes = [ctypes.c_float, i32]
    lib.oracle_key.restype = ctypes.c_uint64
    _lib = lib
    return lib


def metric_code(metric):
    if isinstance(metric, str):
        return _METRICS[metric]
    return int(metric)


def _ptr(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def brute_force_knn(base, queries, k, metric="l2", threads=0):
    """Exact k-NN (src/knn.cpp:71-142) on the CPU, float32 math."""
    lib = _load()
    base = np.ascontiguousarray(base, dtype=np.float32)
    queries = np.ascontiguousarray(queries, dtype=np.float32)
    n, d = base.shape
    nq = queries.shape[0]
    ids = np.empty((nq, k), np.int32)
    dist = np.empty((nq, k), np.float32)
    rc = lib.oracle_brute_force_knn(
        _ptr(base), n, _ptr(queries), nq, d, k, metric_code(metric),
        _ptr(ids), _ptr(dist), threads)
    if rc != 0:
        raise ValueError("oracle: invalid argument")
    return ids, dist


def knn_keys(base, queries, k, metric="l2", id_offset=0, threads=0):
    """The k best 64-bit (score, id) keys per query, best first."""
    lib = _load()
    base = np.ascontiguousarray(base, dtype=np.float32)
    queries = np.ascontiguousarray(queries, dtype=np.float32)
    n, d = base.shape
    nq = queries.shape[0]
    keys = np.empty((nq, k), np.uint64)
    rc = lib.oracle_knn_keys(
        _ptr(base), n, _ptr(queries), nq, d, k, metric_code(metric),
        id_offset, _ptr(keys), threads)
    if rc != 0:
        raise ValueError("oracle: invalid argument")
    return keys


def hamming_knn(rows, queries, k, threads=0):
    """Exact Hamming k-NN of bit-packed uint8 rows (src/ivf.cpp:1343-1403)."""
    lib = _load()
    rows = np.ascontiguousarray(rows, dtype=np.uint8)
    queries = np.ascontiguousarray(queries, dtype=np.uint8)
    n, nbytes = rows.shape
    nq = queries.shape[0]
    ids = np.empty((nq, k), np.int32)
    dist = np.empty((nq, k), np.float32)
    rc = lib.oracle_hamming_knn(
        _ptr(rows), n, _ptr(queries), nq, nbytes, k, _ptr(ids), _ptr(dist), threads)
    if rc != 0:
        raise ValueError("oracle: invalid argument")
    return ids, dist


def merge_keys(lists, k):
    """Best k distinct keys of L key lists laid out [L, nq, k] (0 = empty
    slot), best first; a key present in several lists is taken once."""
    lib = _load()
    lists = np.ascontiguousarray(lists, dtype=np.uint64)
    L, nq, kk = lists.shape
    assert kk == k
    out = np.empty((nq, k), np.uint64)
    lib.oracle_merge_keys(_ptr(lists), L, nq, k, _ptr(out))
    return out


def key(score, idx):
    return int(_load().oracle_key(float(score), int(idx)))


def decode_keys(keys):
    """(ids int32, scores float32) of 64-bit keys; 0 decodes to (-1, -inf)."""
    keys = np.asarray(keys, dtype=np.uint64)
    lo = (keys & np.uint64(0xFFFFFFFF)).astype(np.uint32)
    hi = (keys >> np.uint64(32)).astype(np.uint32)
    ids = (~lo).view(np.int32).copy()
    u = np.where(hi & np.uint32(0x80000000), hi ^ np.uint32(0x80000000), ~hi)
    scores = u.astype(np.uint32).view(np.float32).copy()
    empty = keys == 0
    ids[empty] = -1
    scores[empty] = -np.inf
    return ids, scores


def all_neighbors(rows, k, metric="l2", threads=0, begin=0, end=None):
    """Exact k-NN graph, as the reference builds it with algo BruteForce and
    one cluster: brute_force_knn of the rows against themselves with
    min(k + 1, n) neighbors (src/all_neighbors.cpp:250-263), then
    merge_lists (:56-95): entries that are -1 or the row itself are dropped,
    the rest ordered by distance (nearest first; ties keep the id order of
    the argsort by id, i.e. lower id first), the best k kept, -1 / +-inf
    padding.  begin / end: the lists of those rows only."""
    rows = np.ascontiguousarray(rows, dtype=np.float32)
    n = rows.shape[0]
    end = n if end is None else end
    kk = min(k + 1, n)
    ids, dist = brute_force_knn(rows, rows[begin:end], kk, metric, threads)
    l2 = metric_code(metric) == L2
    key = (dist if l2 else -dist).astype(np.float64)
    dropped = (ids < 0) | (ids == np.arange(begin, end, dtype=np.int64)[:, None])
    key[dropped] = np.inf
    out_ids = np.full((end - begin, k), -1, np.int32)
    out_dist = np.full((end - begin, k), np.inf if l2 else -np.inf, np.float32)
    for i in range(end - begin):
        by_id = np.argsort(ids[i], kind="stable")
        sid, skey, sdist = ids[i][by_id], key[i][by_id], dist[i][by_id]
        repeat = np.concatenate([[False], sid[1:] == sid[:-1]])
        skey = np.where(repeat, np.inf, skey)
        best = np.argsort(skey, kind="stable")[:k]
        kept = skey[best] < np.inf
        m = len(best)
        out_ids[i, :m] = np.where(kept, sid[best], -1)
        out_dist[i, :m] = np.where(kept, sdist[best], out_dist[i, :m])
    return out_ids, out_dist


def _order_bits(v):
    """The sign-flip map of src/kernels.h:16-19 (float32 -> uint32, order kept)."""
    u = np.ascontiguousarray(v, dtype=np.float32).view(np.uint32).astype(np.uint64)
    return np.where(u & 0x80000000, (~u) & 0xFFFFFFFF, u | 0x80000000)


def topk_merge(scores, ids, best, id_offset, first, k):
    """One merge step (src/knn.cpp:37-69, kernel src/kernels.h:37-229): per
    row, the k largest (score key, then lower id as unsigned) of the t new
    entries (ids id_offset + column) and, unless first, the k running ones;
    then ordered by score (float compare) and id; -1 / -inf padding."""
    scores = np.asarray(scores, dtype=np.float32)
    nq, t = scores.shape
    out_ids = np.full((nq, k), -1, np.int32)
    out_sc = np.full((nq, k), -np.inf, np.float32)
    for i in range(nq):
        v = scores[i]
        idv = (id_offset + np.arange(t, dtype=np.int64)).astype(np.int32)
        if not first:
            v = np.concatenate([v, np.asarray(best[i], np.float32)])
            idv = np.concatenate([idv, np.asarray(ids[i], np.int32)])
        key = (_order_bits(v) << np.uint64(32)) | (~idv.view(np.uint32)).astype(np.uint64)
        take = np.argsort(key, kind="stable")[::-1][:k]
        sv, si = v[take], idv[take]
        order = np.lexsort((si.view(np.uint32), -sv.astype(np.float64)))
        m = len(take)
        out_ids[i, :m] = si[order]
        out_sc[i, :m] = sv[order]
    return out_ids, out_sc


def refine(dataset, queries, candidates, k, metric="l2"):
    """Exact re-ranking (src/ivf.cpp:1642-1708): float32 scores of each
    candidate row (L2 -sum((r - q)^2), inner product, cosine on unit rows),
    -inf for ids outside [0, n); the k best by a stable sort on -score
    (equal scores keep the candidates' order); infinite scores are missing
    (-1, +inf for L2, -inf otherwise)."""
    ds = np.asarray(dataset, dtype=np.float32)
    q = np.asarray(queries, dtype=np.float32)
    cand = np.asarray(candidates).astype(np.int64)
    n = ds.shape[0]
    valid = (cand >= 0) & (cand < n)
    rows = ds[np.where(valid, cand, 0)]
    code = metric_code(metric)
    qq = q[:, None, :]
    if code == COSINE:
        rows = rows / np.maximum(np.sqrt((rows * rows).sum(2, keepdims=True)), np.float32(1e-30))
        qq = qq / np.maximum(np.sqrt((qq * qq).sum(2, keepdims=True)), np.float32(1e-30))
    if code == L2:
        score = -((rows - qq) ** 2).sum(2, dtype=np.float32)
    else:
        score = (rows * qq).sum(2, dtype=np.float32)
    score = np.where(valid, score, -np.inf).astype(np.float32)
    order = np.argsort(-score, axis=1, kind="stable")[:, :k]
    best = np.take_along_axis(score, order, 1)
    missing = np.isinf(best)
    ids = np.where(missing, -1, np.take_along_axis(cand, order, 1)).astype(np.int32)
    if code == L2:
        dist = np.where(missing, np.inf, -best)
    else:
        dist = np.where(missing, -np.inf, best)
    return ids, dist.astype(np.float32)
