"""The IVF list scan on the tensor cores (csrc/ivftc.cu) against the oracle:
search ids and score bits identical to ivf.rs's per-list search and merge
(restated in the oracle), with the tensor-core path forced on (tuning key
ivf_tc 2) and checked to have run (its launches counted, no CUDA-core list
scan), over centered and uncentered lists, widths 64..2048, 1..4 bits, k 1
to 32, one to every list probed; lists longer than a 512-record range, more
than 128 pairs on one list, lists shorter than k, duplicated records (exact
ties), zero queries, and a store overflow that must fall back to the
CUDA-core scan with the same results."""
from __future__ import annotations

import numpy as np
import pytest

from test_gpu_ivf import bits_equal, clustered, oracle_lists

pytestmark = pytest.mark.gpu


def run_tc(uv, fn):
    """fn() with the tensor-core list scan forced on; returns (result, tc
    scan launches, CUDA-core list scan launches)."""
    uv.set_tuning("ivf_tc", 2)
    uv.profile_enable(True)
    try:
        out = fn()
        tc = uv.profile_read("ivf_tc_scan")[1]
        cc = uv.profile_read("ivf_scan")[1]
    finally:
        uv.profile_enable(False)
        uv.set_tuning("ivf_tc", 0)
    return out, tc, cc


def build(oracle, uv, n, nq, dim, bits, mem, nlist, centered, seed, iters=3):
    rows = clustered(n + nq, dim, 10, seed)
    base, queries = rows[:n], rows[n:] * np.float32(1.3)
    cen = oracle.kmeans(base, nlist, seed=42, iters=iters)
    assign = oracle.assign(base, cen)
    ocodec = oracle.Codec(dim, bits, mem)
    off, ids, lists = oracle_lists(oracle, ocodec, base, cen, assign, centered)
    ivf = uv.IvfIndex(uv.Codec(dim, bits, mem), cen, centered=centered)
    ivf.build(base, assign=assign)
    return base, queries, cen, ocodec, off, ids, lists, ivf


@pytest.mark.parametrize("centered", [True, False])
@pytest.mark.parametrize("dim,bits,mem,nlist", [(64, 2, 6, 12), (256, 2, 8, 16), (96, 3, 5, 9),
                                                (128, 1, 8, 10), (128, 4, 6, 10),
                                                (2048, 2, 8, 6)])
def test_tensor_core_list_scan_bit_exact(oracle, uv, centered, dim, bits, mem, nlist):
    n = 1200 if dim == 2048 else 2500
    nq = 24
    base, queries, cen, ocodec, off, ids, lists, ivf = build(
        oracle, uv, n, nq, dim, bits, mem, nlist, centered, dim + bits * 7 + nlist)
    queries[3] = 0.0  # a zero query: k unfilled slots
    for nprobe in (1, 3, nlist):
        for k in (1, 10, 32):
            (gi, gs), tc, cc = run_tc(uv, lambda: ivf.search(queries, k, nprobe))
            assert tc == 1 and cc == 0, (nprobe, k, tc, cc)
            wi, ws = ocodec.ivf_search_topk(cen, off, ids, lists, centered, queries, nprobe, k)
            assert np.array_equal(gi, wi), (nprobe, k)
            assert bits_equal(gs, ws), (nprobe, k)
            assert (gi[3] == -1).all() and np.isneginf(gs[3]).all()


def test_long_lists_many_pairs_short_lists(oracle, uv):
    """Two big lists (ranges of 512 records: 3 and more per list), 300
    queries on 3 lists (more than 128 pairs per list), and a list of 4
    records (fewer than k)."""
    dim, bits, mem = 128, 2, 8
    n, nq = 3004, 300
    rows = clustered(n + nq, dim, 2, 5)
    base, queries = rows[:n], rows[n:]
    cen = oracle.kmeans(base[:3000], 2, seed=42, iters=2)
    far = base[3000:].copy()
    far[:] = -cen[0] - cen[1]
    far /= np.linalg.norm(far, axis=1, keepdims=True)
    far += np.float32(1e-3) * np.arange(4, dtype=np.float32)[:, None]
    base[3000:] = far
    cen = np.concatenate([cen, far[:1]])
    assign = oracle.assign(base, cen)
    assert np.bincount(assign, minlength=3).min() >= 1
    for centered in (True, False):
        ocodec = oracle.Codec(dim, bits, mem)
        off, ids, lists = oracle_lists(oracle, ocodec, base, cen, assign, centered)
        assert (np.diff(off)[:2] > 1024).all()
        ivf = uv.IvfIndex(uv.Codec(dim, bits, mem), cen, centered=centered)
        ivf.build(base, assign=assign)
        for k, nprobe in [(10, 3), (32, 2), (5, 1), (16, 3)]:
            (gi, gs), tc, cc = run_tc(uv, lambda: ivf.search(queries, k, nprobe))
            assert tc == 1 and cc == 0
            wi, ws = ocodec.ivf_search_topk(cen, off, ids, lists, centered, queries, nprobe, k)
            assert np.array_equal(gi, wi), (centered, k, nprobe)
            assert bits_equal(gs, ws), (centered, k, nprobe)


def test_one_long_list_many_ranges(oracle, uv):
    """60,000 records in one list: 118 ranges of 512, each with its own
    threshold, so thousands of lower bounds reach the largest range
    threshold and the query threshold comes from the radix select; the
    search stays on the tensor cores and matches the oracle."""
    dim, bits, mem = 64, 2, 6
    rows = clustered(60_008, dim, 3, 23)
    base, queries = rows[:60_000], rows[60_000:]
    cen = oracle.kmeans(base, 1, seed=42, iters=1)
    assign = np.zeros(len(base), np.uint32)
    for centered in (True, False):
        ocodec = oracle.Codec(dim, bits, mem)
        off, ids, lists = oracle_lists(oracle, ocodec, base, cen, assign, centered)
        ivf = uv.IvfIndex(uv.Codec(dim, bits, mem), cen, centered=centered)
        ivf.build(base, assign=assign)
        for k in (10, 32):
            (gi, gs), tc, cc = run_tc(uv, lambda: ivf.search(queries, k, 1))
            assert tc == 1 and cc == 0, (centered, k)
            wi, ws = ocodec.ivf_search_topk(cen, off, ids, lists, centered, queries, 1, k)
            assert np.array_equal(gi, wi), (centered, k)
            assert bits_equal(gs, ws), (centered, k)


def test_duplicates_ties_and_overflow_fallback(oracle, uv):
    """Duplicated records tie exactly (ranked by id); 40 copies keep every
    copy through the bounds and stay on the tensor-core path; 1200 copies of
    one record overflow a query's store and the search reruns on the
    CUDA-core scan -- the same results either way."""
    dim, bits, mem, nlist = 64, 2, 6, 4
    for copies, expect_fallback in [(40, False), (1200, True)]:
        rows = clustered(1500, dim, 4, 17 + copies)
        base, queries = rows[:1400].copy(), rows[1400:]
        base[100:100 + copies] = base[99]
        base = np.concatenate([base, np.repeat(base[99:100], max(0, copies - 1300), axis=0)])
        cen = oracle.kmeans(base, nlist, seed=42, iters=3)
        assign = oracle.assign(base, cen)
        ocodec = oracle.Codec(dim, bits, mem)
        off, ids, lists = oracle_lists(oracle, ocodec, base, cen, assign, True)
        ivf = uv.IvfIndex(uv.Codec(dim, bits, mem), cen, centered=True)
        ivf.build(base, assign=assign)
        q = np.concatenate([queries, base[99:100] * np.float32(2.0)])
        (gi, gs), tc, cc = run_tc(uv, lambda: ivf.search(q, 10, 2))
        assert tc == 1 and (cc == 1) == expect_fallback, (copies, tc, cc)
        wi, ws = ocodec.ivf_search_topk(cen, off, ids, lists, True, q, 2, 10)
        assert np.array_equal(gi, wi), copies
        assert bits_equal(gs, ws), copies


def test_automatic_choice_and_off_switch(oracle, uv):
    """ivf_tc 0 takes the tensor-core scan for rows of 256 or more
    coordinates and k <= 32; ivf_tc 1 never; both give the oracle's results."""
    dim, bits, mem, nlist = 256, 2, 8, 8
    base, queries, cen, ocodec, off, ids, lists, ivf = build(
        oracle, uv, 1500, 16, dim, bits, mem, nlist, True, 3)
    wi, ws = ocodec.ivf_search_topk(cen, off, ids, lists, True, queries, 2, 10)
    for mode, want_tc in [(0, 1), (1, 0)]:
        uv.set_tuning("ivf_tc", mode)
        uv.profile_enable(True)
        try:
            gi, gs = ivf.search(queries, 10, 2)
            tc = uv.profile_read("ivf_tc_scan")[1]
        finally:
            uv.profile_enable(False)
            uv.set_tuning("ivf_tc", 0)
        assert tc == want_tc
        assert np.array_equal(gi, wi) and bits_equal(gs, ws)
    with pytest.raises(uv.UVError):
        uv.set_tuning("ivf_tc", 3)
