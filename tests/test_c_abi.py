"""The C ABI library on the CPU: it loads, exports every function the header
declares, and maps bad arguments to MLXVS_ERROR_INVALID_ARGUMENT with the
reference's messages (src/c_api.cpp:30-47,84-91) before touching a GPU."""

import ctypes
import os
import re
import threading

import numpy as np
import pytest

import mlxvs_b200 as mv

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "mlxvs_c.h")


def declared_functions():
    text = open(HEADER).read()
    return re.findall(r"MLXVS_C_API\s+[\w\s\*]+?\b(mlxvs_\w+)\s*\(", text)


@pytest.fixture(scope="module")
def lib():
    if not os.path.exists(mv.library_path()):
        from mlxvs_b200 import build

        build.build()
    return mv._load()


def test_exports_every_declared_function(lib):
    names = declared_functions()
    assert len(names) >= 12
    raw = ctypes.CDLL(mv.library_path())
    for name in names:
        assert hasattr(raw, name), name


def test_exports_nothing_else():
    import subprocess

    out = subprocess.run(["nm", "-D", "--defined-only", mv.library_path()],
                         capture_output=True, text=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    # the C++ API of include/mlxvs.h (namespace mlxvs) is checked in test_cpp_api
    exported = {s for s in exported if not s.startswith("_ZN5mlxvs")}
    assert exported == set(declared_functions())


def test_version_and_empty_error(lib):
    assert mv.version()
    assert lib.mlxvs_last_error() == b""


def call_knn(lib, base, n, queries, nq, d, k, metric, ids, dist):
    return lib.mlxvs_brute_force_knn(base, n, queries, nq, d, k, metric, ids, dist)


def test_argument_errors(lib):
    b = np.zeros((4, 3), np.float32)
    ids = np.zeros((2, 5), np.int32)
    dist = np.zeros((2, 5), np.float32)
    p = lambda a: a.ctypes.data
    cases = [
        ((p(b), 4, p(b), 2, 3, 5, 1, None, p(dist)), b"ids must not be NULL"),
        ((None, 4, p(b), 2, 3, 5, 1, p(ids), p(dist)), b"rows must not be NULL"),
        ((p(b), -1, p(b), 2, 3, 5, 1, p(ids), p(dist)), b"[0, 2^31)"),
        ((p(b), 4, p(b), 2, 0, 5, 1, p(ids), p(dist)), b"dimension must be at least 1"),
        ((p(b), 4, p(b), 2, 3, 300, 1, p(ids), p(dist)), b"k must be in [1, 256]"),
        ((p(b), 4, p(b), 2, 3, 0, 1, p(ids), p(dist)), b"k must be in [1, 256]"),
        ((p(b), 4, p(b), 2, 3, 5, 7, p(ids), p(dist)), b"unknown metric"),
    ]
    for args, msg in cases:
        assert call_knn(lib, *args) == 1
        assert msg in lib.mlxvs_last_error(), (args, lib.mlxvs_last_error())
    codes = np.zeros((4, 16), np.uint8)
    assert lib.mlxvs_hamming_knn(p(codes), 4, p(codes), 2, 16, 300, p(ids), p(dist)) == 1
    assert b"k must be in [1, 256]" in lib.mlxvs_last_error()
    assert lib.mlxvs_hamming_knn(p(codes), 4, p(codes), 2, 0, 3, p(ids), p(dist)) == 1


def test_python_errors_are_value_errors(lib):
    with pytest.raises(ValueError, match="same number of columns"):
        mv.brute_force_knn(np.zeros((4, 3)), np.zeros((2, 5)), 1)
    with pytest.raises(ValueError, match="k must be in"):
        mv.brute_force_knn(np.zeros((4, 3)), np.zeros((2, 3)), 300)
    with pytest.raises(ValueError, match="real numbers"):
        mv.brute_force_knn(np.zeros((4, 3), bool), np.zeros((2, 3)), 1)
    with pytest.raises(ValueError, match="2-D"):
        mv.brute_force_knn(np.zeros(4), np.zeros((2, 3)), 1)
    with pytest.raises(ValueError, match="unknown Metric 'cosin'"):
        mv.brute_force_knn(np.zeros((4, 3)), np.zeros((2, 3)), 1, "cosin")
    with pytest.raises(ValueError, match="bit-packed uint8"):
        mv.hamming_knn(np.zeros((4, 3), np.int32), np.zeros((2, 3), np.uint8), 1)


def test_last_error_is_per_thread(lib):
    b = np.zeros((4, 3), np.float32)
    assert call_knn(lib, b.ctypes.data, 4, b.ctypes.data, 2, 3, 300, 1, None, None) == 1
    seen = []
    t = threading.Thread(target=lambda: seen.append(mv._load().mlxvs_last_error()))
    t.start()
    t.join()
    assert seen == [b""]
    assert lib.mlxvs_last_error() != b""


def test_no_gpu_fails_loudly(lib):
    try:
        import torch

        if torch.cuda.is_available():
            pytest.skip("a GPU is present")
    except ImportError:
        pass
    b = np.ones((8, 4), np.float32)
    ids = np.zeros((2, 3), np.int32)
    dist = np.zeros((2, 3), np.float32)
    rc = call_knn(lib, b.ctypes.data, 8, b.ctypes.data, 2, 4, 3, 1, ids.ctypes.data,
                  dist.ctypes.data)
    assert rc == 3
    assert b"CUDA" in lib.mlxvs_last_error()
    with pytest.raises(RuntimeError):
        mv.brute_force_knn(b, b[:2], 3)


def test_exchange_argument_errors(lib):
    # the peer exchange's set-up checks its arguments before any CUDA call
    p = ctypes.c_void_p()
    assert lib.mlxvs_exchange_create(9, 0, 100, ctypes.byref(p)) == 1
    assert b"world must be in [1, 8]" in lib.mlxvs_last_error()
    assert lib.mlxvs_exchange_create(2, 2, 100, ctypes.byref(p)) == 1
    assert lib.mlxvs_exchange_create(2, 0, 0, ctypes.byref(p)) == 1
    assert lib.mlxvs_exchange_create(2, 0, 100, None) == 1
    assert lib.mlxvs_exchange_keys(None, 1, ctypes.byref(p)) == 1
    assert lib.mlxvs_exchange_merge_device(None, 1, 10, 10, 1, None, 0, None, None, None) == 1
    assert lib.mlxvs_exchange_destroy(None) == 0
