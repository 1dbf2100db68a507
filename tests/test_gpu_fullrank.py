"""search(q, limit) for any limit, and rows of any width, on the GPU against
the oracle.

The reference's search scores every entry, sorts and truncates to `limit`
(src/trellis.rs:2120-2183), and its MIPS harness asks for limit = len() and
re-ranks all of them by the row norm (src/bench.rs:1029-1045).  Above the
fused top-k capacity (128) the library ranks every record (scan kernel in
full-ranking mode, then a segmented merge sort); the whole sorted list must
equal the oracle's, ids and score bits, ties by id.

TrellisQuantizer accepts any dimension, and lut_dot_u32 finishes with a
scalar tail (src/simd.rs:240-243): widths that are not a multiple of 16 run
the decode-GEMM over the 16- and 8-wide blocks and add the last d % 8
products one at a time, in order."""
from __future__ import annotations

import numpy as np
import pytest

from fixtures import rand_rows

pytestmark = pytest.mark.gpu


def _bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def _index(uv, dim, bits, mem, rows, centroids=None):
    g = uv.Codec(dim, bits, mem)
    ix = uv.Index(g)
    if centroids is not None:
        ix.set_centroids(centroids)
    ix.add_batch(rows)
    return g, ix


def _check(ix, o, enc, qs, k, norms):
    ids, scores = ix.search(qs, k, mips=norms is not None)
    wids, wscores = o.search_topk(enc, qs, k, norms=norms)
    np.testing.assert_array_equal(ids, wids)
    np.testing.assert_array_equal(_bits(scores), _bits(wscores))
    return ids, scores


@pytest.mark.parametrize("mips", [True, False])
def test_limit_equal_to_len_matches_the_oracle(uv, oracle, mips):
    """The MIPS harness's call: search(q, db.len()) on a 10k index."""
    n = 10_000
    rows = rand_rows(n, 128, 21)
    qs = rand_rows(24, 128, 22)
    g, ix = _index(uv, 128, 2, 8, rows)
    o = oracle.Codec(128, 2, 8)
    enc = o.encode_batch(rows)
    norms = oracle.l2_norms(rows) if mips else None
    ids, scores = _check(ix, o, enc, qs, n, norms)
    # every record exactly once per query, in ranking order
    assert (np.sort(ids, axis=1) == np.arange(n)).all()
    assert (np.diff(scores, axis=1) <= 0).all()


@pytest.mark.parametrize("k", [129, 300, 2049, 5000])
def test_k_above_the_fused_capacity(uv, oracle, k):
    """Merge passes that keep only the best k of each run (k below, at and
    above the 2048-entry sort tile), over 20k records."""
    rows = rand_rows(20_000, 64, 31)
    qs = rand_rows(9, 64, 32)
    g, ix = _index(uv, 64, 2, 8, rows)
    o = oracle.Codec(64, 2, 8)
    enc = o.encode_batch(rows)
    _check(ix, o, enc, qs, k, oracle.l2_norms(rows))
    _check(ix, o, enc, qs, k, None)


def test_full_ranking_edge_cases(uv, oracle):
    """k > len (unfilled slots), a degenerate query, exact ties broken by id
    (duplicate rows), a zero row (rescale +inf, score 0), an odd width and a
    length that is not a multiple of the sort tile."""
    dim = 72
    rows = rand_rows(4099, dim, 41)
    rows[7] = rows[3]
    rows[1000] = rows[3]
    rows[20] = 0.0
    qs = rand_rows(6, dim, 42)
    qs[2] = 0.0
    g, ix = _index(uv, dim, 2, 8, rows)
    o = oracle.Codec(dim, 2, 8)
    enc = o.encode_batch(rows)
    for norms in (None, oracle.l2_norms(rows)):
        ids, scores = _check(ix, o, enc, qs, 5000, norms)
        assert (ids[2] == -1).all() and np.isneginf(scores[2]).all()
        assert (ids[0, 4099:] == -1).all()


def test_full_ranking_centered_and_wide_rows(uv, oracle):
    """A centered index (qm per centroid) and rows wider than 384 (the
    K-chunked scan kernel in full-ranking mode)."""
    rows = oracle.rand_unit(3000, 128, 51)
    qs = oracle.rand_unit(7, 128, 52)
    cen = oracle.kmeans(rows, 4, 42)
    g, ix = _index(uv, 128, 2, 8, rows, centroids=cen)
    o = oracle.Codec(128, 2, 8, centroids=cen)
    enc = o.encode_batch(rows)
    _check(ix, o, enc, qs, 3000, None)

    rows = rand_rows(2500, 512, 53)
    qs = rand_rows(5, 512, 54)
    g, ix = _index(uv, 512, 2, 8, rows)
    o = oracle.Codec(512, 2, 8)
    enc = o.encode_batch(rows)
    _check(ix, o, enc, qs, 700, oracle.l2_norms(rows))


def test_full_ranking_device_buffers(uv, oracle):
    """Device queries and outputs (written in place, chunk by chunk)."""
    import torch

    rows = rand_rows(3000, 128, 61)
    qs = rand_rows(11, 128, 62)
    g, ix = _index(uv, 128, 2, 8, rows)
    ids_d, sc_d = ix.search(torch.from_numpy(qs).cuda(), 3000, mips=True)
    torch.cuda.synchronize()
    ids_h, sc_h = ix.search(qs, 3000, mips=True)
    np.testing.assert_array_equal(ids_d.cpu().numpy(), ids_h)
    np.testing.assert_array_equal(_bits(sc_d.cpu().numpy()), _bits(sc_h))


@pytest.mark.parametrize("dim,bits,mem", [(100, 2, 8), (72, 2, 8), (37, 1, 8), (130, 3, 6),
                                          (12, 2, 8), (8, 4, 5), (420, 2, 8), (600, 1, 8),
                                          (1001, 2, 8)])
def test_flat_search_any_width(uv, oracle, dim, bits, mem):
    """Widths with an 8-wide block and/or a scalar tail, resident-query and
    K-chunked kernels (above 384), MIPS and cosine, k = 10 and 100."""
    rows = rand_rows(1200, dim, 3 * dim + bits)
    qs = rand_rows(33, dim, 3 * dim + bits + 1)
    g, ix = _index(uv, dim, bits, mem, rows)
    o = oracle.Codec(dim, bits, mem)
    enc = o.encode_batch(rows)
    ex = ix.export()
    np.testing.assert_array_equal(ex["codes"], enc["codes"])
    for norms in (None, oracle.l2_norms(rows)):
        for k in (10, 100):
            _check(ix, o, enc, qs, k, norms)


def test_ivf_search_any_width(uv, oracle):
    """The IVF list scan over rows whose width has a scalar tail."""
    from test_gpu_ivf import clustered, oracle_lists, bits_equal

    n, nq, dim, nlist = 1500, 20, 100, 9
    rows = clustered(n + nq, dim, 6, 77)
    base, queries = rows[:n], rows[n:]
    cen = oracle.kmeans(base, nlist, seed=42, iters=3)
    assign = oracle.assign(base, cen)
    for centered in (False, True):
        ocodec = oracle.Codec(dim, 2, 8)
        off, ids, lists = oracle_lists(oracle, ocodec, base, cen, assign, centered)
        ivf = uv.IvfIndex(uv.Codec(dim, 2, 8), cen, centered=centered)
        ivf.build(base)
        for nprobe in (1, 4):
            gi, gs = ivf.search(queries, 10, nprobe)
            wi, ws = ocodec.ivf_search_topk(cen, off, ids, lists, centered, queries, nprobe, 10)
            assert np.array_equal(gi, wi)
            assert bits_equal(gs, ws)
