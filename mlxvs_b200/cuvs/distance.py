"""cuVS's distance vocabulary (``cuvs.distance``) as the brute-force front end
needs it: the ``cuvs::distance::DistanceType`` numbers (they are written into
index files, so they keep cuVS's values), the metric names and their
conversion from this library's scores.

Follows python/mlxvs/cuvs/distance.py:11-56 (the enum and the name table) and
python/mlxvs/cuvs/neighbors/_common.py:39-52 (scores to cuVS distances).
"""

import numpy as np

__all__ = ["DISTANCE_NAMES", "DISTANCE_TYPES", "metric_type", "to_cuvs_distances"]

# cuvs::distance::DistanceType
L2Expanded = 0
L2SqrtExpanded = 1
CosineExpanded = 2
L1 = 3
L2Unexpanded = 4
L2SqrtUnexpanded = 5
InnerProduct = 6
Linf = 7
Canberra = 8
LpUnexpanded = 9
CorrelationExpanded = 10
JaccardExpanded = 11
HellingerExpanded = 12
Haversine = 13
BrayCurtis = 14
JensenShannon = 15
HammingUnexpanded = 16
KLDivergence = 17
RusselRaoExpanded = 18
DiceExpanded = 19
BitwiseHamming = 20

DISTANCE_TYPES = {
    "l2": L2SqrtExpanded,
    "sqeuclidean": L2Expanded,
    "euclidean": L2SqrtExpanded,
    "l1": L1,
    "cityblock": L1,
    "inner_product": InnerProduct,
    "chebyshev": Linf,
    "canberra": Canberra,
    "cosine": CosineExpanded,
    "lp": LpUnexpanded,
    "correlation": CorrelationExpanded,
    "jaccard": JaccardExpanded,
    "hellinger": HellingerExpanded,
    "braycurtis": BrayCurtis,
    "jensenshannon": JensenShannon,
    "hamming": HammingUnexpanded,
    "kl_divergence": KLDivergence,
    "minkowski": LpUnexpanded,
    "russellrao": RusselRaoExpanded,
    "dice": DiceExpanded,
    "bitwise_hamming": BitwiseHamming,
}

DISTANCE_NAMES = {v: k for k, v in DISTANCE_TYPES.items()}

# The DistanceTypes the sm_100a search computes, with the Metric each runs as.
# Every other type is an elementwise metric that this library does not run.
FAST = {
    L2Expanded: "l2",
    L2SqrtExpanded: "l2",
    InnerProduct: "inner_product",
    CosineExpanded: "cosine",
}


def metric_type(metric):
    """A metric name (any key of DISTANCE_TYPES) or DistanceType number as the
    DistanceType number; an unknown name raises ValueError."""
    if isinstance(metric, str):
        if metric not in DISTANCE_TYPES:
            raise ValueError(f"metric {metric} is not supported")
        return DISTANCE_TYPES[metric]
    return int(metric)


def is_min_close(distance_type):
    """Smaller distances are closer for every type but the inner product."""
    return distance_type != InnerProduct


def to_cuvs_distances(scores, distance_type):
    """This library's scores (squared L2, inner product, cosine similarity)
    as the distances cuVS returns for ``distance_type``: the square root of
    the clamped squared distance for the Sqrt types, the clamped squared
    distance for the others of L2, 1 - similarity for cosine, the inner
    product as it is.  ``scores`` is a float32 numpy array or torch tensor;
    the result has the same kind."""
    is_np = type(scores).__module__ == "numpy"
    if distance_type in (L2SqrtExpanded, L2SqrtUnexpanded, L2Expanded, L2Unexpanded):
        s = np.maximum(scores, np.float32(0)) if is_np else scores.clamp_min(0)
        if distance_type in (L2SqrtExpanded, L2SqrtUnexpanded):
            s = np.sqrt(s) if is_np else s.sqrt()
        return s
    if distance_type == CosineExpanded:
        return 1 - scores
    return scores
