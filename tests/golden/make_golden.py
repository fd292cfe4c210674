"""Writes tests/golden/golden.json: small seeded cases with their expected
outputs, from the CPU oracle (oracle/oracle.c) and the reference's own
known-answer tests.

The reference (MLX + Metal) cannot run on Linux, so no output of it is
recorded here; the integer-valued and Hamming cases are exact arithmetic
(any correct implementation must give these ids and distances), the
float case is the oracle's float32 result.

Run from the repository root:  python tests/golden/make_golden.py
"""

import json
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from oracle import oracle as O  # noqa: E402
from tests import data  # noqa: E402

CASES = [
    {"name": "mixture-l2-k10", "metric": "l2", "k": 10,
     "input": {"kind": "mixture", "n": 3000, "d": 128, "clusters": 16, "seed": 11, "nq": 8}},
    {"name": "mixture-ip-k5", "metric": "inner_product", "k": 5,
     "input": {"kind": "mixture", "n": 2000, "d": 64, "clusters": 8, "seed": 12, "nq": 6}},
    {"name": "mixture-l2-k33-ties", "metric": "l2", "k": 33,
     "input": {"kind": "mixture", "n": 1500, "d": 8, "clusters": 4, "seed": 13, "nq": 4}},
    {"name": "normal-cosine-k10", "metric": "cosine", "k": 10, "exact": False,
     "input": {"kind": "normal", "n": 1000, "d": 48, "seed": 21, "nq": 4}},
    {"name": "hamming-32B-k10", "k": 10,
     "input": {"kind": "hamming", "n": 5000, "bytes": 32, "prototypes": 40, "flip": 0.1,
               "seed": 7, "nq": 6}},
    {"name": "hamming-128B-k12", "k": 12,
     "input": {"kind": "hamming", "n": 3000, "bytes": 128, "prototypes": 64, "flip": 0.1,
               "seed": 8, "nq": 5}},
]


def main():
    out = []
    for case in CASES:
        spec = case["input"]
        if spec["kind"] == "mixture":
            b, q = data.gaussian_mixture_int(spec["n"], spec["d"], spec["clusters"], spec["seed"],
                                             nq=spec["nq"])
            ids, dist = O.brute_force_knn(b, q, case["k"], case["metric"])
        elif spec["kind"] == "normal":
            b = data.normal_rows(spec["n"], spec["d"], spec["seed"])
            q = data.normal_rows(spec["nq"], spec["d"], spec["seed"] + 1)
            ids, dist = O.brute_force_knn(b, q, case["k"], case["metric"])
        else:
            b, q = data.hamming_codes(spec["n"], spec["bytes"], spec["prototypes"], spec["flip"],
                                      spec["seed"], nq=spec["nq"])
            ids, dist = O.hamming_knn(b, q, case["k"])
        out.append(dict(case, ids=ids.tolist(), distances=[[float(v) for v in r] for r in dist]))
    # the reference's own known-answer tests, verbatim expectations
    out.append({"name": "kat-ties (tests/test_knn.cpp:158-192)", "metric": "l2", "k": 10,
                "input": {"kind": "ties"},
                "ids": [[w for w in range(1, 12) if w % 97 != 0][:10]] * 2,
                "distances": [[0.0] * 10] * 2})
    out.append({"name": "kat-hamming-tiny (python/tests/test_cuvs.py:844-849)", "k": 2,
                "input": {"kind": "hamming-tiny"}, "ids": [[0, 1]], "distances": [[0.0, 3.0]]})
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden.json")
    with open(path, "w") as f:
        json.dump(out, f, separators=(",", ":"))
    print(path, os.path.getsize(path), "bytes")


if __name__ == "__main__":
    main()
