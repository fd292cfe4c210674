"""Builds libmlxvs_b200.so in-tree with nvcc for sm_100a.

Usage: python -m mlxvs_b200.build [--verbose]
The library exports the C API of include/mlxvs_c.h and the C++ API of
include/mlxvs.h (the rest is hidden).
"""

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libmlxvs_b200.so")
SOURCES = ["engine.cu", "c_api.cpp", "cpp_api.cu"]
HEADERS = ["common.cuh", "gemm_topk.cuh", "gemm_topk_q.cuh", "hamming.cuh", "knn_kernels.cuh",
           "select.cuh", "engine.h"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path():
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def flags(extra=()):
    return [
        *ARCH,
        "-O3",
        "-lineinfo",
        "-std=c++17",
        "--expt-relaxed-constexpr",
        "-Xcompiler",
        "-fPIC,-fvisibility=hidden,-O3",
        "-I",
        os.path.join(ROOT, "include"),
        "-I",
        CSRC,
        *extra,
    ]


def stale():
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    deps = [os.path.join(CSRC, f) for f in SOURCES + HEADERS]
    deps += [os.path.join(ROOT, "include", h) for h in ("mlxvs_c.h", "mlxvs.h")]
    return any(os.path.getmtime(p) > t for p in deps)


def build(verbose=False, force=False, extra=()):
    """Compiles the library unless it is up to date; returns its path."""
    if not force and not stale():
        return LIB
    nvcc = nvcc_path()
    # The environment may point the host compiler at a wrapper; nvcc uses
    # the system g++ by default, which is what we want.
    env = dict(os.environ)
    env.pop("NVCC_PREPEND_FLAGS", None)
    env.pop("NVCC_APPEND_FLAGS", None)
    tmp = LIB + ".tmp"
    cmd = [nvcc, *flags(extra), "-shared", "-o", tmp] + [os.path.join(CSRC, f) for f in SOURCES]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True, env=env, cwd=CSRC)
    os.replace(tmp, LIB)
    return LIB


def ptxas_report():
    """Registers / spills / shared memory per kernel (nvcc -Xptxas -v)."""
    nvcc = nvcc_path()
    cmd = [nvcc, *flags(["-Xptxas", "-v"]), "-c", "-o", os.devnull, os.path.join(CSRC, "engine.cu")]
    out = subprocess.run(cmd, capture_output=True, text=True, cwd=CSRC)
    return out.stdout + out.stderr


if __name__ == "__main__":
    if "--ptxas" in sys.argv:
        print(ptxas_report())
    else:
        print(build(verbose="--verbose" in sys.argv, force="--force" in sys.argv))
