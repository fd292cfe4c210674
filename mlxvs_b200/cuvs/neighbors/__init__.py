"""cuVS's ``cuvs.neighbors`` for the exact search: ``brute_force``."""

from mlxvs_b200.cuvs.neighbors import brute_force

__all__ = ["brute_force"]
