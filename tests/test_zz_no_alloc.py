"""mlxvs_hamming_knn_noalloc: the Hamming search for callers that cannot
allocate device memory (a serving loop that must not stall other streams,
since cudaMalloc and cudaFree synchronize the device; a process whose
framework already holds the GPU's memory; code with a fixed footprint after
start-up).  Its scratch is a static 16 MiB array inside the library, shared
by every call.

These tests call it through the C ABI and require the same ids and
distances as the allocating entry point (bit for bit: Hamming distances are
integers), over consecutive calls on different inputs, so that anything the
previous call left in the shared array would show.  This file is collected
last, so a run that stops at the first failure has run every other test.
"""

import ctypes

import numpy as np
import pytest

import mlxvs_b200 as mv
from tests import data

pytestmark = pytest.mark.gpu


def noalloc_entry():
    lib = mv._load()
    fn = lib.mlxvs_hamming_knn_noalloc
    p, i64, i32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32
    fn.argtypes = [p, i64, p, i64, i32, i32, p, p, p]
    fn.restype = ctypes.c_int
    return lib, fn


def run_noalloc(fn, rows, queries, k):
    import torch

    nq = queries.shape[0]
    ids = torch.full((nq, k), -7, dtype=torch.int32, device=queries.device)
    dist = torch.full((nq, k), float("nan"), dtype=torch.float32, device=queries.device)
    stream = torch.cuda.current_stream(queries.device).cuda_stream
    rc = fn(rows.data_ptr(), rows.shape[0], queries.data_ptr(), nq, rows.shape[1], k,
            ids.data_ptr(), dist.data_ptr(), ctypes.c_void_p(stream))
    return rc, ids, dist


def test_matches_allocating_entry_point_on_consecutive_calls():
    import torch

    lib, fn = noalloc_entry()
    cases = [
        data.hamming_codes(60_000, 128, 4096, 0.1, seed=21, nq=700) + (10,),
        data.hamming_codes(33_333, 64, 512, 0.15, seed=22, nq=257) + (25,),
        data.hamming_codes(60_000, 128, 4096, 0.1, seed=21, nq=700) + (10,),
    ]
    for rows_np, q_np, k in cases:
        rows = torch.from_numpy(rows_np).cuda()
        q = torch.from_numpy(q_np).cuda()
        want_ids, want_dist = mv.hamming_knn(rows, q, k)
        rc, ids, dist = run_noalloc(fn, rows, q, k)
        assert rc == 0, lib.mlxvs_last_error()
        torch.cuda.synchronize()
        assert torch.equal(ids, want_ids)
        assert torch.equal(dist, want_dist)


def test_widest_codes_and_a_list_array_that_fills_the_scratch():
    # 512-byte codes (the widest it reads in place, 128 queries per block),
    # and nq * k so large that the scratch holds the lists of one base range
    # only (the array, not the work, sets the number of ranges); two calls
    # in a row each
    import torch

    lib, fn = noalloc_entry()
    cases = [
        data.hamming_codes(5_000, 512, 256, 0.1, seed=23, nq=300) + (10,),
        data.hamming_codes(20_000, 16, 2048, 0.1, seed=24, nq=50_000) + (32,),
    ]
    for rows_np, q_np, k in cases:
        rows = torch.from_numpy(rows_np).cuda()
        q = torch.from_numpy(q_np).cuda()
        want_ids, want_dist = mv.hamming_knn(rows, q, k)
        for _ in range(2):
            rc, ids, dist = run_noalloc(fn, rows, q, k)
            assert rc == 0, lib.mlxvs_last_error()
            torch.cuda.synchronize()
            assert torch.equal(ids, want_ids)
            assert torch.equal(dist, want_dist)


def test_rejects_what_it_cannot_do_without_allocating():
    import torch

    lib, fn = noalloc_entry()
    rows = torch.zeros((100, 48), dtype=torch.uint8, device="cuda")
    rc, _, _ = run_noalloc(fn, rows, rows[:4], 5)
    assert rc == 1 and b"bytes must be" in lib.mlxvs_last_error()
    rows = torch.zeros((100, 16), dtype=torch.uint8, device="cuda")
    big = torch.zeros((400_000, 16), dtype=torch.uint8, device="cuda")
    rc, _, _ = run_noalloc(fn, rows, big, 10)
    assert rc == 1 and b"16 MiB" in lib.mlxvs_last_error()
    rc, ids, _ = run_noalloc(fn, rows, rows[:3], 4)
    assert rc == 0, lib.mlxvs_last_error()
    torch.cuda.synchronize()
    assert ids.shape == (3, 4) and np.all(ids.cpu().numpy()[:, 0] >= 0)
