"""The C++ API of include/mlxvs.h (mlxvs::brute_force_knn, hamming_knn,
topk_merge; ref include/mlxvs/mlxvs.h:59-65,780-784,898-905), called from a
C++ program (tests/cpp/test_cpp_api.cpp) built against the in-tree library.

On the CPU: the library exports every declared C++ function and the
program's argument checks pass (they raise before any GPU work).  On a GPU:
the program runs every entry on host and on device arrays (which must give
the same bytes) and writes its inputs and results, checked here against the
oracle -- bit-exact for the integer-valued inputs, float tolerance for cosine.
"""

import os
import re
import shutil
import subprocess

import numpy as np
import pytest

import mlxvs_b200 as mv
from oracle import oracle as O

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "mlxvs.h")
SOURCE = os.path.join(ROOT, "tests", "cpp", "test_cpp_api.cpp")
CUDA = "/usr/local/cuda"


def declared_cpp_functions():
    text = open(HEADER).read()
    return re.findall(r"MLXVS_CPP_API\s+[\w:<>,\s\*&]+?\b(\w+)\s*\(", text)


@pytest.fixture(scope="module")
def program(tmp_path_factory):
    if not os.path.exists(mv.library_path()):
        from mlxvs_b200 import build

        build.build()
    cxx = shutil.which("g++")
    if cxx is None:
        pytest.skip("no C++ compiler")
    exe = str(tmp_path_factory.mktemp("cpp") / "test_cpp_api")
    libdir = os.path.dirname(mv.library_path())
    cmd = [cxx, "-std=c++17", "-O1", "-Wall", "-Werror", "-I", os.path.join(ROOT, "include"),
           "-I", os.path.join(CUDA, "include"), SOURCE, "-o", exe, "-L", libdir, "-lmlxvs_b200",
           "-L", os.path.join(CUDA, "lib64"), "-lcudart", f"-Wl,-rpath,{libdir}",
           f"-Wl,-rpath,{os.path.join(CUDA, 'lib64')}"]
    subprocess.run(cmd, check=True)
    return exe


def test_exports_every_declared_cpp_function():
    names = declared_cpp_functions()
    assert set(names) == {"dtype_size", "brute_force_knn", "hamming_knn", "topk_merge"}
    out = subprocess.run(["nm", "-D", "--defined-only", "-C", mv.library_path()],
                         capture_output=True, text=True, check=True).stdout
    exported = {m.group(1) for m in re.finditer(r" T mlxvs::(\w+)\(", out)}
    assert exported == set(names)


def test_argument_errors(program):
    r = subprocess.run([program, "errors"], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0, r.stderr
    assert r.stdout.strip() == "ok"


def load(d, name, dtype, shape):
    return np.fromfile(os.path.join(d, name), dtype=dtype).reshape(shape)


@pytest.mark.gpu
def test_every_entry_on_host_and_device_arrays(program, tmp_path):
    from tests.test_gpu_knn import check_float

    r = subprocess.run([program, "run", str(tmp_path)], capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0, r.stderr
    n, nq, d, nc, nqc, nbytes, t = 3000, 37, 64, 5000, 41, 32, 500
    base = load(tmp_path, "base.f32", np.float32, (n, d))
    queries = load(tmp_path, "queries.f32", np.float32, (nq, d))
    for metric, name in (("inner_product", "ip"), ("l2", "l2"), ("cosine", "cosine")):
        ids = load(tmp_path, f"knn_{name}.ids", np.int32, (nq, 10))
        dist = load(tmp_path, f"knn_{name}.dist", np.float32, (nq, 10))
        if metric == "cosine":
            check_float(metric, base, queries, 10, ids, dist)
        else:
            oids, odist = O.brute_force_knn(base, queries, 10, metric)
            assert np.array_equal(ids, oids), name
            assert np.array_equal(dist, odist), name
    ids = load(tmp_path, "few.ids", np.int32, (nq, 8))
    dist = load(tmp_path, "few.dist", np.float32, (nq, 8))
    oids, odist = O.brute_force_knn(base[:5], queries, 8, "l2")
    assert np.array_equal(ids, oids) and (ids[:, 5:] == -1).all()
    assert np.array_equal(dist, odist) and np.isposinf(dist[:, 5:]).all()

    codes = load(tmp_path, "codes.u8", np.uint8, (nc, nbytes))
    qcodes = load(tmp_path, "qcodes.u8", np.uint8, (nqc, nbytes))
    oids, odist = O.hamming_knn(codes, qcodes, 16)
    assert np.array_equal(load(tmp_path, "hamming.ids", np.int32, (nqc, 16)), oids)
    assert np.array_equal(load(tmp_path, "hamming.dist", np.float32, (nqc, 16)), odist)

    s1 = load(tmp_path, "scores.f32", np.float32, (nq, t))
    s2 = load(tmp_path, "scores2.f32", np.float32, (nq, t))
    i1, v1 = O.topk_merge(s1, None, None, 0, True, 8)
    assert np.array_equal(load(tmp_path, "merge1.ids", np.int32, (nq, 8)), i1)
    assert np.array_equal(load(tmp_path, "merge1.scores", np.float32, (nq, 8)), v1)
    i2, v2 = O.topk_merge(s2, i1, v1, t, False, 8)
    assert np.array_equal(load(tmp_path, "merge2.ids", np.int32, (nq, 8)), i2)
    assert np.array_equal(load(tmp_path, "merge2.scores", np.float32, (nq, 8)), v2)
