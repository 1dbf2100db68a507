"""The coset trellis on the GPU (coset.cu, capi_coset.cu, the coset decoder
of scan.cu) against the oracle (oracle/uv_oracle_coset.c): books, records
(start state + packed symbols, rescale, rnorm, centroid) and search results
bit-identical, through the C ABI."""
from __future__ import annotations

import numpy as np
import pytest

from fixtures import rand_rows

pytestmark = pytest.mark.gpu


def _same_f32(a, b):
    return np.array_equal(np.asarray(a, np.float32).view(np.uint32),
                          np.asarray(b, np.float32).view(np.uint32))


def _pair(uv, oracle, dim, bits, mem, centroids=None):
    g = uv.CosetIndex(dim, bits, mem=mem)
    o = oracle.Coset(dim, bits, mem=mem, centroids=centroids)
    if centroids is not None:
        g.set_centroids(centroids)
    return g, o


@pytest.mark.parametrize("bits", [1, 2])
def test_books_match_oracle(uv, oracle, bits):
    g, o = _pair(uv, oracle, 16, bits, 4)
    keys, scale = g.books()
    assert np.array_equal(keys, o.books())
    assert scale == o.scale()


@pytest.mark.parametrize("dim,bits,mem,n", [
    (64, 2, 12, 300),    # the reference's default memory
    (24, 1, 1, 200),     # mem 1: the 2-state window rule; dim % 16 == 8
    (32, 1, 2, 200),
    (128, 2, 6, 257),
    (40, 2, 13, 64),     # costs still in shared memory
    (64, 1, 14, 48),     # costs in global memory
    (16, 1, 17, 24),     # back pointers in global memory too
])
def test_records_match_oracle(uv, oracle, dim, bits, mem, n):
    g, o = _pair(uv, oracle, dim, bits, mem)
    rows = rand_rows(n, dim, dim * 7 + mem)
    rows[3] = 0.0                       # zero row: |x| clamped at EPS
    rows[5] *= np.float32(1e-30)        # tiny row
    rows[7] = 1.0                       # constant and one-hot rows: tied minima
    rows[9] = 0.0
    rows[9, 0] = 1.0
    g.add_batch(rows)
    got = g.export()
    want = o.encode_batch(rows)
    assert np.array_equal(got["codes"], want["codes"])
    assert _same_f32(got["rescale"], want["rescale"])
    assert _same_f32(got["rnorm"], want["rnorm"])
    assert np.array_equal(got["cidx"], want["cidx"])
    assert np.array_equal(got["ids"], np.arange(n))


@pytest.mark.parametrize("mode", [0, 1], ids=["book_scan", "reference_search"])
def test_nearest_modes_agree(uv, oracle, mode):
    """Both ways to the nearest kept point (tuning key coset_nearest) give
    the oracle's records, tied minima included."""
    uv.set_tuning("coset_nearest", mode)
    try:
        g, o = _pair(uv, oracle, 48, 2, 8)
        rows = rand_rows(150, 48, 77)
        rows[::10] = np.round(rows[::10])  # integer rows: more exact ties
        g.add_batch(rows)
        got = g.export()
        want = o.encode_batch(rows)
        assert np.array_equal(got["codes"], want["codes"])
        assert _same_f32(got["rescale"], want["rescale"])
    finally:
        uv.set_tuning("coset_nearest", 0)


def test_records_three_bits(uv, oracle):
    """2^21 points per coset: the bisection + ball search at three bits."""
    g, o = _pair(uv, oracle, 16, 3, 4)
    rows = rand_rows(12, 16, 33)
    g.add_batch(rows)
    got = g.export()
    want = o.encode_batch(rows)
    assert np.array_equal(got["codes"], want["codes"])
    assert _same_f32(got["rescale"], want["rescale"])


def test_centered_records_and_search(uv, oracle):
    dim = 32
    rng = np.random.default_rng(4)
    cen = rng.standard_normal((5, dim)).astype(np.float32) * np.float32(0.2)
    g, o = _pair(uv, oracle, dim, 2, 8, centroids=cen)
    rows = rand_rows(400, dim, 21)
    g.add_batch(rows)
    got = g.export()
    want = o.encode_batch(rows)
    assert np.array_equal(got["codes"], want["codes"])
    assert _same_f32(got["rnorm"], want["rnorm"])
    assert np.array_equal(got["cidx"], want["cidx"])
    q = rand_rows(40, dim, 22)
    ids, sc = g.search(q, 17)
    wids, wsc = o.search(want, q, 17)
    assert np.array_equal(ids, wids) and _same_f32(sc, wsc)


@pytest.mark.parametrize("dim,bits,mem,n,k", [
    (64, 2, 12, 3000, 10),
    (24, 1, 3, 1500, 100),    # padded lanes of the last 8-wide block
    (128, 2, 8, 5000, 128),
    (512, 1, 6, 700, 32),     # rows too wide for the flat tile: K-chunked scan
    (64, 2, 12, 3000, 3000),  # k = n: every record ranked (full ranking above 128)
    (24, 1, 3, 1500, 200),
    (512, 1, 6, 700, 701),    # K-chunked scan, k past n: the tail unfilled
])
def test_search_matches_oracle(uv, oracle, dim, bits, mem, n, k):
    g, o = _pair(uv, oracle, dim, bits, mem)
    rows = rand_rows(n, dim, n + dim)
    g.add_batch(rows)
    want = o.encode_batch(rows)
    q = rand_rows(70, dim, 5)
    q[1] = 0.0  # zero query: clamped, every score 0, insertion order
    ids, sc = g.search(q, k)
    wids, wsc = o.search(want, q, k)
    assert np.array_equal(ids, wids)
    assert _same_f32(sc, wsc)


def test_ids_ties_and_short_index(uv, oracle):
    """add_batch numbers each batch 0..n-1 (the reference's add_batch);
    add keeps given ids; equal records tie in insertion order; k above the
    index size leaves id -1 / -inf."""
    dim = 32
    g, o = _pair(uv, oracle, dim, 2, 6)
    rows = rand_rows(50, dim, 8)
    g.add_batch(rows)
    g.add_batch(rows[:10])
    g.add(np.arange(1000, 1005), rows[:5])
    ex = g.export()
    assert list(ex["ids"][:50]) == list(range(50))
    assert list(ex["ids"][50:60]) == list(range(10))
    assert list(ex["ids"][60:]) == list(range(1000, 1005))
    ids, sc = g.search(rows[:3], 3)
    for qi in range(3):
        assert list(ids[qi]) == [qi, qi, 1000 + qi]
        assert sc[qi, 0] == sc[qi, 1] == sc[qi, 2]
    small = uv.CosetIndex(dim, 2, mem=6)
    small.add_batch(rows[:4])
    ids, sc = small.search(rows[:2], 6)
    assert list(ids[0, 4:]) == [-1, -1] and np.all(np.isneginf(sc[:, 4:]))


def test_reconstruct_matches_oracle(uv, oracle):
    dim = 64
    g, o = _pair(uv, oracle, dim, 2, 12)
    v = np.array([((j * 37) % 101) / 101.0 - 0.5 for j in range(dim)], np.float32)
    rows = np.concatenate([v[None], rand_rows(7, dim, 9)])
    out = g.reconstruct(rows)
    for i in range(len(rows)):
        assert _same_f32(out[i], o.reconstruct_unit(rows[i]))
    assert float(v @ out[0]) / np.linalg.norm(v) > 0.5


def test_sizes_and_refusals(uv, oracle):
    g, o = _pair(uv, oracle, 128, 2, 12)
    g.add_batch(rand_rows(10, 128, 1))
    assert len(g) == 10
    assert g.code_len == o.code_len == 32
    assert g.mem_bytes() == o.mem_bytes(10)
    assert g.model_bytes() == 3 * 128 * 4 + 8 * 8192 * 16
    with pytest.raises(uv.UVError):
        g.set_centroids(np.zeros((2, 128), np.float32))  # after the first add
    for dim, bits, mem in [(12, 2, 4), (16, 0, 4), (16, 4, 4), (16, 2, 0), (16, 2, 21)]:
        with pytest.raises(uv.UVError):
            uv.CosetIndex(dim, bits, mem=mem)
    with pytest.raises(uv.UVError):
        g.search(rand_rows(2, 128, 3), 0)
    ids, sc = g.search(rand_rows(2, 128, 3), 129)  # any k: the tail unfilled
    assert (ids[:, 10:] == -1).all() and (ids[:, :10] >= 0).all()


def test_device_tensors(uv, oracle):
    import torch

    dim = 64
    g, o = _pair(uv, oracle, dim, 2, 10)
    rows = rand_rows(800, dim, 12)
    g.add_batch(torch.from_numpy(rows).cuda())
    want = o.encode_batch(rows)
    q = torch.from_numpy(rand_rows(33, dim, 13)).cuda()
    ids, sc = g.search(q, 20)
    assert ids.is_cuda and sc.is_cuda
    wids, wsc = o.search(want, q.cpu().numpy(), 20)
    assert np.array_equal(ids.cpu().numpy(), wids)
    assert _same_f32(sc.cpu().numpy(), wsc)
