"""The search half of cuVS's ``cuvs.neighbors.brute_force`` API (``build``
and ``search``), routed to this library's sm_100a exact search.

It stands in for the branches of python/mlxvs/cuvs/neighbors/brute_force.py:98-116
that call the reference's ``brute_force_knn`` and ``hamming_knn``.  Metric
routing:

* ``sqeuclidean``, ``euclidean``/``l2``, ``inner_product`` and ``cosine`` go to
  :func:`mlxvs_b200.brute_force_knn`, whose scores are then turned into cuVS
  distances;
* ``bitwise_hamming`` (rows of bit-packed uint8) goes to
  :func:`mlxvs_b200.hamming_knn`;
* every other cuVS metric, and any real prefilter, raises NotImplementedError:
  the library has no kernel for them and computes nothing on the host.

Index files (cuVS ``save``/``load``) are not part of this library.

Where the work runs: on the GPU of the dataset when it is a CUDA tensor (else
of the queries, when they are), returning CUDA tensors; for host inputs,
through the host-memory entry, returning numpy arrays.
"""

import numpy as np

import mlxvs_b200 as _mv
from mlxvs_b200.cuvs import distance as _d

__all__ = ["Index", "build", "search"]


class Index:
    """What ``build`` returns: a reference to the rows plus the metric to
    search them with."""

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
    """Wraps ``dataset`` as an index for :func:`search`; nothing is computed
    (an exact search needs no structure beyond the rows).

    Args:
        dataset: ``[n, dim]`` rows.  Float rows for the float metrics,
          bit-packed uint8 rows for ``"bitwise_hamming"``.  A CUDA tensor is
          kept on its device; other inputs are kept as numpy arrays.
        metric (str | int): a metric name from ``cuvs.distance`` or its
          DistanceType number.
        metric_arg (float): kept on the index (only ``"minkowski"`` uses it,
          and that metric is not searched here).
        resources: ignored; the work is queued on the current CUDA stream of
          the device that holds the rows.

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
    """Exact k nearest neighbors of each query row among the index rows.

    Args:
        index (Index): from :func:`build`.
        queries: ``[n_queries, dim]`` rows of the same kind as the dataset.
        k (int): 1 .. 256.  Slots past the number of rows hold id -1 and an
          infinite distance (negative infinity for ``inner_product``).
        neighbors: optional preallocated ``[n_queries, k]`` array or tensor
          that receives the ids.
        distances: optional preallocated ``[n_queries, k]`` array or tensor
          that receives the distances.
        resources: ignored.
        prefilter: None, or a filter whose ``type`` is ``"none"``.

    Returns:
        tuple: ``(distances, neighbors)`` as float32 and int64, each row in
        increasing distance, equal distances ordered by row id.
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

