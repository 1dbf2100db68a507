"""Batched CandidateScorer / PreparedQuery (csrc/candidates.cu, csrc/capi_cand.cu)
against the oracle (trellis.rs:2016-2086): every score bit-identical, on
ragged CSR batches, centered indexes, zero queries, odd dimensions, host and
device buffers; positions outside the index and malformed offsets refused."""
from __future__ import annotations

import numpy as np
import pytest

from fixtures import rand_rows

pytestmark = pytest.mark.gpu


def oracle_records(index):
    e = index.export()
    return dict(codes=e["codes"], start=e["start"], rescale=e["rescale"], rnorm=e["rnorm"])


def ragged_batch(nq, n_rec, seed, max_len=300):
    rng = np.random.default_rng(seed)
    lens = rng.integers(0, max_len, nq)
    lens[0] = 0  # an empty list
    off = np.zeros(nq + 1, np.int64)
    off[1:] = np.cumsum(lens)
    pos = rng.integers(0, n_rec, int(off[-1])).astype(np.int64)  # duplicates included
    return off, pos


def same_bits(a, b):
    a, b = np.asarray(a, np.float32), np.asarray(b, np.float32)
    assert a.shape == b.shape
    bad = np.nonzero(a.view(np.uint32) != b.view(np.uint32))[0]
    assert bad.size == 0, f"{bad.size} scores differ, first at {bad[:5]}: {a[bad[:5]]} vs {b[bad[:5]]}"


@pytest.fixture(params=[0, 1], ids=["lane", "halfwarp"])
def kernel(uv, request):
    """Both scorer kernels: one thread per candidate (bits 1, 2, 4) and half a
    warp per candidate (every width)."""
    uv.set_tuning("cand_kernel", request.param)
    yield request.param
    uv.set_tuning("cand_kernel", 0)


@pytest.mark.parametrize("dim,bits,mem", [(128, 2, 8), (64, 1, 12), (128, 4, 6), (128, 3, 7),
                                          (256, 1, 14), (96, 2, 10)])
def test_batched_scores_bit_exact(uv, oracle, kernel, dim, bits, mem):
    rows = rand_rows(6000, dim, 51) * np.float32(2.5)
    queries = rand_rows(48, dim, 52)
    queries[7] = 0.0  # degenerate: every candidate scores 0.0
    codec = uv.Codec(dim, bits, mem)
    index = uv.Index(codec)
    index.add_batch(rows)
    off, pos = ragged_batch(48, 6000, 53)
    prep = index.prepare(queries)
    assert len(prep) == 48
    got = prep.score(pos, off)
    ref = oracle.Codec(dim, bits, mem).score_candidates(oracle_records(index), queries, pos, off)
    same_bits(got, ref)
    assert np.all(got[off[7]:off[8]] == 0.0)


def test_centered_index_and_odd_dims(uv, oracle, kernel):
    for dim in (40, 44, 100):
        rows = rand_rows(2000, dim, 54)
        queries = rand_rows(12, dim, 55)
        cen = oracle.kmeans(rows, 8, 42)
        codec = uv.Codec(dim, 2, 8)
        index = uv.Index(codec)
        index.set_centroids(cen)
        index.add_batch(rows)
        off, pos = ragged_batch(12, 2000, 56, 200)
        got = index.prepare(queries).score(pos, off)
        ocodec = oracle.Codec(dim, 2, 8, centroids=cen)
        enc = ocodec.encode_batch(rows)
        recs = oracle_records(index)
        assert np.array_equal(enc["codes"], recs["codes"])
        recs["cidx"] = enc["cidx"]
        ref = ocodec.score_candidates(recs, queries, pos, off)
        same_bits(got, ref)


def test_one_query_forms_agree_with_search(uv, oracle):
    rows = rand_rows(3000, 128, 57)
    q = rand_rows(1, 128, 58)
    codec = uv.Codec(128, 2, 8)
    index = uv.Index(codec)
    index.add_batch(rows)
    allpos = np.arange(3000, dtype=np.int64)
    a = index.score_candidates(q[0], allpos)
    b = index.prepare(q).score(allpos)
    same_bits(a, b)
    # search's top-k scores are the scorer's scores of those records
    ids, scores = index.search(q, 20)
    same_bits(a[ids[0]], scores[0])
    assert float(index.prepare(q).score_at(int(ids[0, 0]))) == float(scores[0, 0])
    assert index.scored_len() == 3000
    table = (1 << (8 + 2)) * 4
    assert index.scorer_model_bytes() >= table + 3 * 128 * 4


def test_device_buffers(uv, oracle):
    import torch

    rows = rand_rows(4000, 128, 59)
    queries = rand_rows(32, 128, 60)
    codec = uv.Codec(128, 2, 8)
    index = uv.Index(codec)
    index.add_batch(torch.from_numpy(rows).cuda())
    off, pos = ragged_batch(32, 4000, 61)
    prep = index.prepare(torch.from_numpy(queries).cuda())
    got = prep.score(torch.from_numpy(pos).cuda(), torch.from_numpy(off).cuda())
    assert got.is_cuda
    ref = oracle.Codec(128, 2, 8).score_candidates(oracle_records(index), queries, pos, off)
    same_bits(got.cpu().numpy(), ref)


def test_large_batch_bit_exact(uv, oracle, kernel):
    """10k candidates per query for 16 queries over 50k records."""
    rows = rand_rows(50_000, 128, 62)
    queries = rand_rows(16, 128, 63)
    codec = uv.Codec(128, 2, 8)
    index = uv.Index(codec)
    index.add_batch(rows)
    rng = np.random.default_rng(64)
    pos = rng.integers(0, 50_000, 16 * 10_000).astype(np.int64)
    off = np.arange(17, dtype=np.int64) * 10_000
    got = index.prepare(queries).score(pos, off)
    ref = oracle.Codec(128, 2, 8).score_candidates(oracle_records(index), queries, pos, off)
    same_bits(got, ref)


def test_bad_positions_and_offsets_are_refused(uv, kernel):
    import torch

    rows = rand_rows(500, 64, 65)
    codec = uv.Codec(64, 2, 6)
    index = uv.Index(codec)
    index.add_batch(rows)
    prep = index.prepare(rand_rows(3, 64, 66))

    def refused(pos, off):
        with pytest.raises(uv.UVError) as e:
            prep.score(pos, off)
        assert e.value.code == 1

    ok_off = np.array([0, 2, 3, 4], np.int64)
    refused(np.array([0, 1, 500, 2], np.int64), ok_off)       # past the end
    refused(np.array([0, -1, 5, 2], np.int64), ok_off)        # negative
    refused(np.array([0, 1, 2, 3], np.int64), np.array([0, 3, 2, 4], np.int64))  # decreasing
    refused(np.array([0, 1, 2, 3], np.int64), np.array([1, 2, 3, 4], np.int64))  # not from 0
    refused(np.array([0, 1, 2, 3], np.int64), None)           # 3 queries need offsets
    # device offsets that do not cover the batch are caught by the kernel
    refused(torch.tensor([0, 1, 2, 3], device="cuda"),
            torch.tensor([0, 1, 2, 3], device="cuda"))
    # the good batch still scores after the refusals
    out = prep.score(np.array([0, 1, 2, 3], np.int64), ok_off)
    assert np.all(np.isfinite(out))
    assert prep.score(np.zeros(0, np.int64), np.zeros(4, np.int64)).shape == (0,)


def test_destroy_order_is_free(uv):
    """A prepared batch may outlive its index, and an index its codec (the
    order a garbage collector picks for a cycle)."""
    codec = uv.Codec(64, 2, 6)
    index = uv.Index(codec)
    index.add_batch(rand_rows(200, 64, 67))
    prep = index.prepare(rand_rows(2, 64, 68))
    index.close()
    prep.close()
    index2 = uv.Index(codec)
    index2.add_batch(rand_rows(50, 64, 69))
    codec.close()
    index2.close()
