"""The tensor-core prefilter of the flat scan (tcscan.cu) returns exactly what
the exact scan returns: ids and scores bit-identical to the oracle at sizes
the oracle finishes in seconds, and to the exact CUDA-core kernel at the full
1M-record size.  `tc_scan` = 2 forces the prefilter wherever it is built,
1 disables it."""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

from fixtures import rand_rows

pytestmark = pytest.mark.gpu

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))


@pytest.fixture(params=[3, 1], ids=["a_tmem", "a_smem"])
def tc_mode(uv, request):
    """Both CTA shapes: the query tile held in TMEM (the default) and in
    shared memory."""
    uv.set_tuning("tc_shape", request.param)
    yield lambda v: uv.set_tuning("tc_scan", v)
    uv.set_tuning("tc_scan", 0)
    uv.set_tuning("tc_shape", 0)


def search_both(uv, index, queries, k, mips, tc_mode):
    tc_mode(2)
    a = index.search(queries, k, mips=mips)
    tc_mode(1)
    b = index.search(queries, k, mips=mips)
    return a, b


def same(a, b):
    return np.array_equal(a[0], b[0]) and np.array_equal(
        np.asarray(a[1], np.float32).view(np.uint32), np.asarray(b[1], np.float32).view(np.uint32))


@pytest.mark.parametrize("rescore", [0, 1], ids=["warp_rescore", "cta_rescore"])
@pytest.mark.parametrize("mips", [True, False])
@pytest.mark.parametrize("k", [10, 100])
def test_matches_oracle(oracle, uv, tc_mode, mips, k, rescore):
    """Both rescoring kernels: one warp per short candidate list (default)
    and one CTA per query everywhere (tuning key rescore_warp = 1)."""
    uv.set_tuning("rescore_warp", rescore)
    n, nq, dim = 70_000, 48, 128
    base = rand_rows(n, dim, 5) * np.float32(2.5)
    base[::7] *= np.float32(0.1)  # spread the norms (MIPS)
    queries = rand_rows(nq, dim, 6)
    ocodec = oracle.Codec(dim, 2, 8)
    enc = ocodec.encode_batch(base)
    want = ocodec.search_topk(enc, queries, k, norms=oracle.l2_norms(base) if mips else None)
    codec = uv.Codec(dim, 2, 8)
    index = uv.Index(codec)
    index.add_batch(base)
    tc_mode(2)
    try:
        got = index.search(queries, k, mips=mips)
    finally:
        uv.set_tuning("rescore_warp", 0)
    assert np.array_equal(got[0], want[0])
    assert np.array_equal(got[1].view(np.uint32), want[1].view(np.uint32))


@pytest.mark.parametrize("bits,mem", [(1, 8), (2, 6), (3, 6), (4, 8), (2, 10)])
def test_code_shapes_match_exact_kernel(uv, tc_mode, bits, mem):
    """Pair table (mem + 2 bits <= 13) and single-value table paths."""
    n, nq, dim = 120_000, 200, 128
    base = rand_rows(n, dim, bits * 10 + mem)
    queries = rand_rows(nq, dim, 99)
    index = uv.Index(uv.Codec(dim, bits, mem))
    index.add_batch(base)
    a, b = search_both(uv, index, queries, 32, True, tc_mode)
    assert same(a, b)


def test_full_size_bench_workload_matches_exact_kernel(uv, tc_mode):
    """1M heavy-tailed, mean-centered rows (the bench generator), k = 100 and
    10, MIPS: identical to the exact kernel."""
    import bench

    base, queries = bench.make_data(1_000_000, 1000)
    index = uv.Index(uv.Codec(128, 2, 8))
    index.add_batch(base)
    for k in (100, 10):
        a, b = search_both(uv, index, queries, k, True, tc_mode)
        assert same(a, b), k


def test_ties_zero_rows_degenerate_queries_ragged_sizes(uv, tc_mode):
    n, nq, dim = 65_537, 131, 128  # neither a multiple of the tile sizes
    base = rand_rows(n, dim, 17)
    base[1000:1400] = base[5]      # exact ties: ranked by record index
    base[2000:2100] = 0.0          # zero rows
    queries = rand_rows(nq, dim, 18)
    queries[3] = 0.0               # degenerate query: empty result
    queries[7] = base[5]
    index = uv.Index(uv.Codec(dim, 2, 8))
    index.add_batch(base)
    for mips in (True, False):
        a, b = search_both(uv, index, queries, 100, mips, tc_mode)
        assert same(a, b), mips
        assert (a[0][3] == -1).all()


def test_all_scores_negative_with_padding_rows(uv, tc_mode):
    """Every MIPS score far below zero and a last tile with padding rows
    (65,537 = 341 tiles of 192 + 65): the padding's zero accumulators must
    not stand in for a record's lower bound, or the threshold would exceed
    every real score and drop the true top-k (one group holds the padding,
    so k = 1 is the case that would show it)."""
    n, nq, dim = 65_537, 40, 128
    base = np.abs(rand_rows(n, dim, 23)) + np.float32(0.1)
    queries = -np.abs(rand_rows(nq, dim, 24)) - np.float32(0.1)
    index = uv.Index(uv.Codec(dim, 2, 8))
    index.add_batch(base)
    for k in (1, 10, 100):
        a, b = search_both(uv, index, queries, k, True, tc_mode)
        assert same(a, b), k
        assert (np.asarray(a[1]) < 0).all() and (np.asarray(a[0]) >= 0).all(), k


def test_candidate_overflow_falls_back_to_the_exact_scan(uv, tc_mode):
    """Every row identical: every record ties with the k-th score, so every
    record is a candidate and the list overflows; the exact scan answers."""
    n, nq, dim = 40_000, 20, 128
    base = np.repeat(rand_rows(1, dim, 3), n, axis=0)
    base[::2] *= np.float32(3.0)
    queries = rand_rows(nq, dim, 4)
    index = uv.Index(uv.Codec(dim, 2, 8))
    index.add_batch(base)
    a, b = search_both(uv, index, queries, 50, True, tc_mode)
    assert same(a, b)


def test_device_tensors(uv, tc_mode):
    import torch

    n, nq, dim = 70_000, 64, 128
    base = rand_rows(n, dim, 8)
    queries = rand_rows(nq, dim, 9)
    index = uv.Index(uv.Codec(dim, 2, 8))
    index.add_batch(torch.from_numpy(base).cuda())
    tc_mode(2)
    ids, sc = index.search(torch.from_numpy(queries).cuda(), 10, mips=True)
    tc_mode(1)
    ids2, sc2 = index.search(queries, 10, mips=True)
    assert np.array_equal(ids.cpu().numpy(), ids2)
    assert np.array_equal(sc.cpu().numpy().view(np.uint32), sc2.view(np.uint32))


@pytest.mark.parametrize("dim", [96, 256, 1024])
@pytest.mark.parametrize("mips", [True, False])
def test_wide_rows_match_oracle(oracle, uv, tc_mode, dim, mips):
    """tcwide.cu: rows of other widths (K streamed in chunks of 64; 96 pads
    to 128) give the oracle's ids and scores bit for bit."""
    n, nq, k = 30_000, 32, 10
    base = rand_rows(n, dim, 17) * np.float32(2.0)
    base[::5] *= np.float32(0.2)
    queries = rand_rows(nq, dim, 18)
    queries[3] = 0.0
    ocodec = oracle.Codec(dim, 2, 8)
    enc = ocodec.encode_batch(base)
    want = ocodec.search_topk(enc, queries, k, norms=oracle.l2_norms(base) if mips else None)
    codec = uv.Codec(dim, 2, 8)
    index = uv.Index(codec)
    index.add_batch(base)
    tc_mode(2)
    got = index.search(queries, k, mips=mips)
    assert np.array_equal(got[0], want[0])
    assert np.array_equal(got[1].view(np.uint32), want[1].view(np.uint32))
    assert np.all(got[0][3] == -1)


def test_wide_rows_large_match_exact_kernel(uv, tc_mode):
    """300k rows of d = 1024 (the wide-row workload's width), top-10 and
    top-100 MIPS: the prefilter and the exact K-chunked scan agree."""
    import torch

    dim = 1024
    rng = np.random.default_rng(19)
    base = torch.from_numpy(rng.random((300_000, dim), dtype=np.float32) +
                            np.float32(0.5) * (np.arange(dim, dtype=np.float32) / np.float32(959)))
    queries = torch.from_numpy(rng.random((200, dim), dtype=np.float32))
    codec = uv.Codec(dim, 2, 8)
    index = uv.Index(codec)
    index.add_batch(base.cuda())
    qd = queries.cuda()
    for k in (10, 100):
        a, b = search_both(uv, index, qd, k, True, tc_mode)
        assert same((a[0].cpu().numpy(), a[1].cpu().numpy()), (b[0].cpu().numpy(), b[1].cpu().numpy()))


def test_kept_rows_follow_every_change_of_the_records(uv, tc_mode):
    """The prefilter's record rows are kept between searches: after an add,
    a clear and a re-add, and a switch between MIPS and cosine, every search
    equals the exact kernel on the records the index holds at that moment,
    and equals a search that makes its rows in scratch (tc_cache 0)."""
    dim, nq, k = 128, 64, 20
    queries = rand_rows(nq, dim, 41)
    index = uv.Index(uv.Codec(dim, 2, 8))
    steps = [("add", rand_rows(60_000, dim, 42)), ("add", rand_rows(30_000, dim, 43) * np.float32(3)),
             ("clear", None), ("add", rand_rows(50_000, dim, 44))]
    try:
        for op, rows in steps:
            if op == "add":
                index.add_batch(rows)
            else:
                index.clear()
                continue
            for mips in (True, False, True):
                a, b = search_both(uv, index, queries, k, mips, tc_mode)
                assert same(a, b)
                tc_mode(2)
                uv.set_tuning("tc_cache", 0)
                c = index.search(queries, k, mips=mips)
                uv.set_tuning("tc_cache", 1)
                assert same(a, c)
    finally:
        uv.set_tuning("tc_cache", 1)


@pytest.mark.parametrize("sample", [1, 5, 16])
@pytest.mark.parametrize("k", [10, 100])
def test_sampled_threshold_matches_exact_kernel(uv, tc_mode, sample, k):
    """Pass 1 bounding every S-th tile (tuning key tc_sample) still returns
    exactly the exact kernel's top-k; S shrinks when the sample would hold
    fewer than 8k groups."""
    n, nq, dim = 300_000, 150, 128
    base = rand_rows(n, dim, 61) * np.float32(1.7)
    queries = rand_rows(nq, dim, 62)
    index = uv.Index(uv.Codec(dim, 2, 8))
    index.add_batch(base)
    uv.set_tuning("tc_sample", sample)
    try:
        a, b = search_both(uv, index, queries, k, True, tc_mode)
    finally:
        uv.set_tuning("tc_sample", 0)
    assert same(a, b)


@pytest.mark.parametrize("bits,mem", [(1, 8), (2, 8), (4, 6), (2, 12)])
def test_row_kernels_agree(uv, bits, mem):
    """The row kernels (tuning key tc_prepare: 0 the shared-memory table
    with |x|^2 summed in f32, 1 the generic kernel, 2 the shared-memory table
    summing in f64) make the same fp16 rows B'.  The f64 sums give the same
    bound constants, hence the same candidates; the f32 sum under its
    rigorous inflation may make a bound constant one fp16 place larger, so
    as many or a few more candidates pass.  Results are the same bits."""
    n, nq, dim = 150_000, 64, 128
    base = rand_rows(n, dim, 70 + bits)
    queries = rand_rows(nq, dim, 71)
    out = []
    try:
        uv.set_tuning("tc_scan", 2)
        for mode in (0, 1, 2):
            uv.set_tuning("tc_prepare", mode)
            index = uv.Index(uv.Codec(dim, bits, mem))
            index.add_batch(base)
            uv.profile_enable(True)
            r = index.search(queries, 50, mips=True)
            cand = uv.profile_read("tc_candidates")[1]
            uv.profile_enable(False)
            out.append((r, cand))
            index.close()
    finally:
        uv.set_tuning("tc_prepare", 0)
        uv.set_tuning("tc_scan", 0)
    assert same(out[0][0], out[1][0])
    assert same(out[2][0], out[1][0])
    assert out[2][1] == out[1][1] > 0
    assert out[1][1] <= out[0][1] <= out[1][1] * 1.01 + 8


@pytest.mark.parametrize("hot", [0, 1, 3, 8])
def test_pass1_sample_choices_give_the_exact_answer(uv, oracle, hot):
    """Pass 1 may bound any subset of the records: the records of largest
    score scale g (tc_hot 0: n/S of them, 3 and 8: n/3 and n/8) or every
    S-th tile (tc_hot 1).  Ids and score bits equal the oracle's either way,
    on heavy-tailed MIPS rows whose norms vary widely."""
    import bench

    base, queries = bench.make_data(150_000, 64)
    codec = uv.Codec(128, 2, 8)
    index = uv.Index(codec)
    index.add_batch(base)
    ex = index.export()
    o = oracle.Codec(128, 2, 8)
    rec = {"codes": ex["codes"], "start": ex["start"], "rescale": ex["rescale"]}
    try:
        uv.set_tuning("tc_hot", hot)
        uv.set_tuning("tc_scan", 2)
        for k in (10, 100):
            ids, scores = index.search(queries, k, mips=True)
            wids, wsc = o.search_topk(rec, queries, k, norms=ex["norms"])
            assert np.array_equal(ids, wids), (hot, k)
            assert np.array_equal(scores.view(np.uint32), wsc.view(np.uint32)), (hot, k)
    finally:
        uv.set_tuning("tc_hot", 0)
        uv.set_tuning("tc_scan", 0)
