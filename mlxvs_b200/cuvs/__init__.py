"""A cuVS-style Python front end (``cuvs.distance``, ``cuvs.neighbors``) of
the exact search, with cuVS's names, arguments and results."""

from mlxvs_b200.cuvs import distance, neighbors

__all__ = ["distance", "neighbors"]
