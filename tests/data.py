"""Seeded synthetic inputs shaped like BASELINE.json's configs (test side, NumPy).

bench.py draws the same distributions on the GPU with torch.
"""

import numpy as np


def gaussian_mixture_int(n, d, clusters, seed, nq=0):
    """Configs 0/1/3: a mixture of isotropic Gaussians (centers ~U[0,100]^d,
    sigma 10), clipped to [0, 255] and rounded: integers stored as float32.
    Returns (base, queries) drawn from the same mixture."""
    rng = np.random.default_rng(seed)
    centers = rng.uniform(0.0, 100.0, (clusters, d))

    def draw(m):
        lab = rng.integers(0, clusters, m)
        x = centers[lab] + 10.0 * rng.standard_normal((m, d))
        return np.rint(np.clip(x, 0.0, 255.0)).astype(np.float32)

    return draw(n), draw(nq)


def lowrank_unit(n, d, rank, seed, nq=0):
    """Config 2: N(0,1) rows plus a shared random rank-`rank` component,
    L2-normalised, float32."""
    rng = np.random.default_rng(seed)
    basis = rng.standard_normal((rank, d))

    def draw(m):
        x = rng.standard_normal((m, d)) + rng.standard_normal((m, rank)) @ basis
        x /= np.linalg.norm(x, axis=1, keepdims=True)
        return x.astype(np.float32)

    return draw(n), draw(nq)


def hamming_codes(n, nbytes, prototypes, flip, seed, nq=0):
    """Config 4: codes of nbytes*8 bits, each a random prototype XOR
    Bernoulli(flip) noise. Returns (rows, queries) uint8."""
    rng = np.random.default_rng(seed)
    protos = rng.integers(0, 256, (prototypes, nbytes), dtype=np.uint8)

    def draw(m):
        lab = rng.integers(0, prototypes, m)
        bits = rng.random((m, nbytes * 8)) < flip
        noise = np.packbits(bits, axis=1, bitorder="little")
        return protos[lab] ^ noise

    return draw(n), draw(nq)


def normal_rows(n, d, seed):
    """python/tests/test_mlxvs.py:9-10: standard normal float32 rows."""
    return np.random.default_rng(seed).standard_normal((n, d), dtype=np.float32)


def exact_scores(metric, q, b):
    """float64 scores of every query against every row; larger is closer
    (python/tests/test_mlxvs.py:13-20)."""
    q = q.astype(np.float64)
    b = b.astype(np.float64)
    if metric == "l2":
        return -(((q[:, None, :] - b[None, :, :]) ** 2).sum(-1))
    if metric == "cosine":
        q = q / np.maximum(np.linalg.norm(q, axis=1, keepdims=True), 1e-30)
        b = b / np.maximum(np.linalg.norm(b, axis=1, keepdims=True), 1e-30)
    return q @ b.T


def recall(ids, scores, k, tol=1e-5):
    """Tie-tolerant recall@k (python/tests/test_mlxvs.py:23-27)."""
    kth = -np.sort(-scores, axis=1)[:, k - 1 : k]
    hit = np.take_along_axis(scores, np.maximum(ids, 0), axis=1) >= kth - tol
    return (hit & (ids >= 0)).sum() / (ids.shape[0] * k)


def ties_rows():
    """tests/test_knn.cpp:158-165: 4000 x 8 rows of 1.0, every 97th row with
    5.0 in its first column; the queries are rows 1 and 2."""
    x = np.ones((4000, 8), np.float32)
    x[::97, 0] = 5.0
    return x, x[1:3].copy()


def golden_inputs(spec):
    """(is_hamming, base, queries) of a tests/golden/golden.json input spec."""
    kind = spec["kind"]
    if kind == "mixture":
        b, q = gaussian_mixture_int(spec["n"], spec["d"], spec["clusters"], spec["seed"],
                                    nq=spec["nq"])
        return False, b, q
    if kind == "normal":
        return False, normal_rows(spec["n"], spec["d"], spec["seed"]), normal_rows(
            spec["nq"], spec["d"], spec["seed"] + 1)
    if kind == "ties":
        b, q = ties_rows()
        return False, b, q
    if kind == "hamming-tiny":
        codes = np.array([[0b1111, 0], [0b1, 0]], dtype=np.uint8)
        return True, codes, codes[:1].copy()
    b, q = hamming_codes(spec["n"], spec["bytes"], spec["prototypes"], spec["flip"], spec["seed"],
                         nq=spec["nq"])
    return True, b, q
