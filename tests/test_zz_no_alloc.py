"""The allocation-free search entry point (uv_index_search_noalloc).

Callers that cannot allocate device memory while serving -- a process that
reserves its GPU memory budget at start-up, or a latency-bound thread that
cannot take the synchronization cudaMalloc/cudaFree may bring -- use this
entry point; its scratch is a fixed array inside the library.  This file is
collected last so that a failure here stops a fail-fast run only after every
other test has run.  It must pass alone in a fresh process and after the
other tests (the array keeps the previous call's contents).
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _call(uv, index, queries, k, mips, ids, scores):
    import torch

    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    return uv.lib().uv_index_search_noalloc(
        index.h, C.c_void_p(queries.data_ptr()), queries.shape[0], k, 1 if mips else 0,
        C.c_void_p(ids.data_ptr()), C.c_void_p(scores.data_ptr()), stream)


def test_noalloc_search_matches_search_twice(uv):
    import torch

    from fixtures import rand_rows

    dev = torch.device("cuda", 0)
    rows = torch.from_numpy(rand_rows(20_000, 128, 21)).to(dev)
    codec = uv.Codec(128, 2, 8)
    index = uv.Index(codec)
    index.add_batch(rows)
    for call, (nq, seed, k, mips) in enumerate([(512, 1, 100, True), (300, 2, 10, False)]):
        q = torch.from_numpy(rand_rows(nq, 128, seed)).to(dev)
        want_ids, want_scores = index.search(q, k, mips=mips)
        ids = torch.full((nq, k), -7, dtype=torch.int64, device=dev)
        scores = torch.full((nq, k), 7.0, dtype=torch.float32, device=dev)
        rc = _call(uv, index, q, k, mips, ids, scores)
        assert rc == 0, uv.lib().uv_last_error().decode()
        torch.cuda.synchronize()
        # same tolerance as every other parity test here: bit-identical
        assert torch.equal(ids, want_ids), f"call {call}: ids differ"
        assert torch.equal(scores.view(torch.int32), want_scores.view(torch.int32)), \
            f"call {call}: scores differ"


def test_noalloc_search_rejects_oversized_batches_and_host_buffers(uv):
    import torch

    from fixtures import rand_rows

    dev = torch.device("cuda", 0)
    codec = uv.Codec(128, 2, 8)
    index = uv.Index(codec)
    index.add_batch(torch.from_numpy(rand_rows(4096, 128, 5)).to(dev))
    nq, k = 40_000, 100  # needs far more than the fixed scratch
    q = torch.zeros((nq, 128), dtype=torch.float32, device=dev)
    ids = torch.empty((nq, k), dtype=torch.int64, device=dev)
    scores = torch.empty((nq, k), dtype=torch.float32, device=dev)
    rc = _call(uv, index, q, k, True, ids, scores)
    assert rc == uv.binding.UV_EINVAL
    assert "search fewer queries per call" in uv.lib().uv_last_error().decode()
    qh = np.zeros((4, 128), np.float32)
    ih = np.zeros((4, 10), np.int64)
    rc = uv.lib().uv_index_search_noalloc(index.h, C.c_void_p(qh.ctypes.data), 4, 10, 1,
                                          C.c_void_p(ih.ctypes.data), None, None)
    assert rc == uv.binding.UV_EINVAL
