"""cuVS's ``cuvs.neighbors.brute_force`` (build, search, save, load) over the
sm_100a exact search of this library.

Follows python/mlxvs/cuvs/neighbors/brute_force.py:14-190.  The metrics the
GPU search computes run there: ``sqeuclidean``, ``euclidean``/``l2``,
``inner_product`` and ``cosine`` through :func:`mlxvs_b200.brute_force_knn`,
and ``bitwise_hamming`` (bit-packed uint8 rows) through
:func:`mlxvs_b200.hamming_knn` -- the re-pointed branches of
brute_force.py:98-116.  The elementwise metrics (l1, chebyshev, canberra, ...)
and prefilters, which the reference computes with a dense pairwise matrix,
are not part of this library: :func:`search` raises NotImplementedError for
them rather than computing anything on the host.

Placement: when the dataset or the queries is a CUDA tensor the search runs
on that GPU (the dataset's, when both are) and returns CUDA tensors;
otherwise it goes through the host entry and returns numpy arrays.
"""

import numpy as np

import mlxvs_b200 as _mv
from mlxvs_b200.cuvs import _records as rec
from mlxvs_b200.cuvs import distance as _d

__all__ = ["Index", "build", "load", "save", "search"]

SERIALIZATION_VERSION = 0
# format version whose half-precision dtype prefix the file uses
_PREFIX_VERSION = 6


class Index:
    """A brute-force index: the dataset and its metric."""

    def __init__(self):
        self.trained = False
        self._dataset = None
        self._metric = _d.L2Expanded
        self._metric_arg = 2.0

    @property
    def dataset(self):
        return self._dataset

    @property
    def metric(self):
        return _d.DISTANCE_NAMES.get(self._metric, self._metric)

    def __len__(self):
        return 0 if self._dataset is None else int(self._dataset.shape[0])

    def __repr__(self):
        return f"Index(type=BruteForce, metric={_d.DISTANCE_NAMES.get(self._metric)})"


def _is_torch(x):
    return type(x).__module__.startswith("torch") and hasattr(x, "is_cuda")


def _rows(x):
    """A CUDA tensor as it is (contiguous); anything else as a numpy array."""
    if _is_torch(x):
        if x.is_cuda:
            return x.contiguous()
        return x.detach().numpy()
    if hasattr(x, "copy_to_host"):
        x = x.copy_to_host()
    return np.ascontiguousarray(np.asarray(x))


def _host(x):
    return x.detach().cpu().numpy() if _is_torch(x) else np.asarray(x)


def _place(data, q):
    """Both operands on the GPU of the CUDA one (the dataset's first), or both
    on the host."""
    if _is_torch(data) or _is_torch(q):
        import torch

        dev = data.device if _is_torch(data) else q.device
        data = data if _is_torch(data) else torch.from_numpy(np.ascontiguousarray(data)).to(dev)
        q = q.to(dev) if _is_torch(q) else torch.from_numpy(np.ascontiguousarray(q)).to(dev)
    return data, q


def _out(array, given):
    """``array`` written into the caller's preallocated ``given`` (a tensor or
    numpy array of the result's shape), else ``array`` itself."""
    if given is None:
        return array
    if _is_torch(given):
        import torch

        src = array if _is_torch(array) else torch.from_numpy(np.asarray(array))
        given.copy_(src.to(device=given.device, dtype=given.dtype))
    else:
        given[...] = _host(array).astype(np.asarray(given).dtype)
    return given


def build(dataset, metric="sqeuclidean", metric_arg=2.0, resources=None):
    """Builds the index of the dataset (it keeps the rows), as cuVS's
    ``brute_force.build``.

    Args:
        dataset: Rows ``[n, dim]`` (a CUDA tensor stays on its GPU), float
          for the float metrics, bit-packed uint8 for ``"bitwise_hamming"``.
        metric (str | int): A name of ``cuvs.distance.DISTANCE_TYPES`` or a
          DistanceType number.
        metric_arg (float): ``p`` of ``"minkowski"`` (kept for the file).
        resources: Accepted for compatibility; the search runs on the
          current CUDA stream of the dataset's device.

    Returns:
        Index
    """
    x = _rows(dataset)
    if x.ndim != 2:
        raise ValueError("dataset must be a matrix")
    idx = Index()
    idx._dataset = x
    idx._metric = _d.metric_type(metric)
    idx._metric_arg = float(metric_arg)
    idx.trained = True
    return idx


def search(index, queries, k, neighbors=None, distances=None, resources=None, prefilter=None):
    """The k nearest rows of every query, as cuVS's ``brute_force.search``.

    Args:
        index (Index): Built by :func:`build` or read by :func:`load`.
        queries: Rows ``[n_queries, dim]`` of the dataset's kind.
        k (int): Neighbors per query, 1 to 256; beyond the dataset's rows the
          lists are padded with id -1 and an infinite distance (minus
          infinity for the inner product).
        neighbors: Optional ``int64 [n_queries, k]`` output, written in place.
        distances: Optional ``float32 [n_queries, k]`` output, written in place.
        resources: Accepted for compatibility.
        prefilter: Only None or a filter of type ``"none"``.

    Returns:
        tuple: ``(distances, neighbors)``, nearest first, ties to the lower
        id; float32 and int64.
    """
    if not index.trained:
        raise ValueError("Index needs to be built before calling search.")
    if prefilter is not None and getattr(prefilter, "type", "none") != "none":
        raise NotImplementedError(
            "prefilters are not supported by the sm_100a brute-force search")
    t = index._metric
    if t != _d.BitwiseHamming and t not in _d.FAST:
        raise NotImplementedError(
            f"metric {_d.DISTANCE_NAMES.get(t, t)} is not computed by this library; the sm_100a "
            "search runs sqeuclidean, euclidean, inner_product, cosine and bitwise_hamming")
    q = _rows(queries)
    if q.ndim != 2:
        raise ValueError("queries must be a matrix")
    data, q = _place(index._dataset, q)
    if t == _d.BitwiseHamming:
        ids, dist = _mv.hamming_knn(data, q, k)
    else:
        ids, scores = _mv.brute_force_knn(data, q, k, _d.FAST[t])
        dist = _d.to_cuvs_distances(scores, t)
    if _is_torch(ids):
        import torch

        ids = ids.to(torch.int64)
        dist = dist.to(torch.float32)
    else:
        ids = ids.astype(np.int64)
        dist = dist.astype(np.float32, copy=False)
    return _out(dist, distances), _out(ids, neighbors)


def save(filename, index, include_dataset=True, resources=None):
    """Saves the index in cuVS's brute-force format (version 0): the dataset's
    dtype prefix, then as NumPy records the version, rows, dim, metric,
    metric_arg, whether the dataset follows, the dataset, whether norms
    follow and the row norms (squared for L2, plain for cosine)."""
    data = np.ascontiguousarray(_host(index._dataset))
    t = index._metric
    with open(filename, "wb") as f:
        f.write(rec.dtype_prefix(data.dtype, _PREFIX_VERSION))
        rec.write_scalar(f, SERIALIZATION_VERSION, np.int32)
        rec.write_scalar(f, data.shape[0], np.uint64)
        rec.write_scalar(f, data.shape[1], np.uint64)
        rec.write_scalar(f, t, np.int32)
        rec.write_scalar(f, index._metric_arg, np.float32)
        rec.write_scalar(f, bool(include_dataset), np.bool_)
        if include_dataset:
            rec.write_array(f, data)
        has_norms = t in (_d.L2Expanded, _d.L2SqrtExpanded, _d.CosineExpanded)
        rec.write_scalar(f, has_norms, np.bool_)
        if has_norms:
            x = data.astype(np.float32)
            norms = np.sum(x * x, axis=1)
            if t == _d.CosineExpanded:
                norms = np.sqrt(norms)
            rec.write_array(f, norms.astype(np.float32))


def load(filename, resources=None):
    """Loads a brute-force index saved by :func:`save` or by cuVS; the dataset
    is a host array (search copies it to the GPU on every call; build an
    index of a CUDA tensor of it to keep it resident)."""
    with open(filename, "rb") as f:
        dtype = rec.read_prefix(f)
        ver = rec.read_scalar(f)
        if ver != SERIALIZATION_VERSION:
            raise ValueError(
                f"serialization version mismatch, expected {SERIALIZATION_VERSION}, got {ver}")
        rows = rec.read_scalar(f)
        dim = rec.read_scalar(f)
        metric = rec.read_scalar(f)
        metric_arg = rec.read_scalar(f)
        if not rec.read_scalar(f):
            raise ValueError("the file holds no dataset; brute force needs it")
        data = rec.read_array(f).astype(dtype, copy=False)
    if data.shape != (rows, dim):
        raise ValueError(f"dataset of shape {data.shape}, the file says ({rows}, {dim})")
    idx = Index()
    idx._dataset = np.ascontiguousarray(data)
    idx._metric = int(metric)
    idx._metric_arg = float(metric_arg)
    idx.trained = True
    return idx
