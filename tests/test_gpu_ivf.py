"""IVF on the GPU against the oracle (ivf.rs, bench.rs:298-349): k-means
centroids, assignments, posting-list records, probes, search and rerank
results -- all bit-identical.

The inputs follow the IVF workload's generator shape (Gaussian centres,
points = centre + 0.3 N(0, 1), renormalized) at sizes the oracle finishes in
seconds."""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def clustered(n, dim, n_centres, seed):
    rng = np.random.default_rng(seed)
    c = rng.standard_normal((n_centres, dim)).astype(np.float32)
    c /= np.linalg.norm(c, axis=1, keepdims=True)
    pick = rng.integers(0, n_centres, n)
    x = c[pick] + np.float32(0.3) * rng.standard_normal((n, dim)).astype(np.float32)
    x /= np.linalg.norm(x, axis=1, keepdims=True)
    return x.astype(np.float32)


def oracle_lists(oracle, ocodec, rows, centroids, assign, centered):
    order = np.argsort(assign, kind="stable")
    off = np.zeros(centroids.shape[0] + 1, np.int64)
    off[1:] = np.cumsum(np.bincount(assign, minlength=centroids.shape[0]))
    enc = ocodec.ivf_encode(rows, centroids if centered else None, assign)
    lists = {k: v[order] for k, v in enc.items()}
    return off, order.astype(np.int64), lists


def bits_equal(a, b):
    return np.array_equal(np.asarray(a, np.float32).view(np.uint32),
                          np.asarray(b, np.float32).view(np.uint32))


@pytest.mark.parametrize("n,dim,nlist,iters", [(3000, 64, 16, 5), (2500, 48, 37, 5),
                                               (1200, 200, 70, 3), (500, 32, 1, 2)])
def test_kmeans_and_assign_bit_exact(oracle, uv, n, dim, nlist, iters):
    rows = clustered(n, dim, 12, n + dim)
    want = oracle.kmeans(rows, nlist, seed=42, iters=iters)
    got = uv.kmeans(rows, nlist, seed=42, iters=iters)
    assert bits_equal(got, want)
    asg_want = oracle.assign(rows, want)
    asg_got = uv.ivf_assign(rows, want)
    assert np.array_equal(asg_got, asg_want)


@pytest.mark.parametrize("n,dim,nlist", [(20_000, 64, 300), (6000, 256, 520)])
def test_tensor_core_kmeans_and_assign_bit_exact(oracle, uv, n, dim, nlist):
    """At 256 or more centroids the assignment runs on the tensor cores
    (fp16 dots, exact dots for the centroids that can still win): k-means
    centroids and assignments stay bit-identical to the oracle, and equal to
    the CUDA-core assignment, duplicated centroids (first maximum) and a zero
    row included."""
    rows = clustered(n, dim, 12, n + dim)
    rows[5] = 0.0
    want = oracle.kmeans(rows, nlist, seed=42, iters=3)
    got = uv.kmeans(rows, nlist, seed=42, iters=3)
    assert bits_equal(got, want)
    cen = want.copy()
    cen[9] = cen[2]  # exact ties: the lower list wins
    asg_want = oracle.assign(rows, cen)
    try:
        asg_got = uv.ivf_assign(rows, cen)
        uv.set_tuning("ivf_tc_probe", 1)
        asg_exact = uv.ivf_assign(rows, cen)
    finally:
        uv.set_tuning("ivf_tc_probe", 0)
    assert np.array_equal(asg_got, asg_want)
    assert np.array_equal(asg_exact, asg_want)
    assert asg_got[5] == 0


def test_assign_ties_pick_the_first_maximum(oracle, uv):
    # duplicated centroids: every dot ties with its twin, the lower index wins;
    # a zero row dots to +-0 everywhere and lands on list 0
    rows = clustered(400, 32, 4, 5)
    rows[7] = 0.0
    cen = clustered(6, 32, 3, 6)
    cen = np.concatenate([cen, cen])
    assert np.array_equal(uv.ivf_assign(rows, cen), oracle.assign(rows, cen))
    assert uv.ivf_assign(rows, cen)[7] == 0


@pytest.mark.parametrize("centered", [False, True])
@pytest.mark.parametrize("dim,bits,mem,nlist", [(64, 2, 6, 12), (128, 2, 8, 24), (96, 3, 5, 9)])
def test_build_records_probe_search_bit_exact(oracle, uv, centered, dim, bits, mem, nlist):
    n, nq = 2000, 40
    rows = clustered(n + nq, dim, 10, dim * 7 + nlist)
    base, queries = rows[:n], rows[n:] * np.float32(1.7)
    cen = oracle.kmeans(base, nlist, seed=42, iters=5)
    assign = oracle.assign(base, cen)
    ocodec = oracle.Codec(dim, bits, mem)
    off, ids, lists = oracle_lists(oracle, ocodec, base, cen, assign, centered)

    codec = uv.Codec(dim, bits, mem)
    ivf = uv.IvfIndex(codec, cen, centered=centered)
    ivf.build(base)  # assignment computed on the device
    assert len(ivf) == n and ivf.nlist == nlist
    ex = ivf.export()
    assert np.array_equal(ex["list_off"], off)
    assert np.array_equal(ex["ids"], ids)
    assert np.array_equal(ex["codes"], lists["codes"])
    assert np.array_equal(ex["start"], lists["start"])
    assert bits_equal(ex["rescale"], lists["rescale"])
    assert bits_equal(ex["rnorm"], lists["rnorm"])
    assert ivf.digest() == oracle.digest(lists["codes"], lists["start"])
    assert ivf.mem_bytes() == n * (codec.code_bytes + codec.start_bytes + codec.rescale_bytes
                                   + (4 if centered else 0))

    for nprobe in (1, 3, nlist):
        got = ivf.probe(queries, nprobe)
        want = np.stack([oracle.ivf_probe(cen, q, nprobe) for q in queries])
        assert np.array_equal(got, want)
        for k in (1, 10, 100):
            gi, gs = ivf.search(queries, k, nprobe)
            wi, ws = ocodec.ivf_search_topk(cen, off, ids, lists, centered, queries, nprobe, k)
            assert np.array_equal(gi, wi), (nprobe, k)
            assert bits_equal(gs, ws), (nprobe, k)


def test_search_wide_rows_and_custom_ids(oracle, uv):
    """d = 1024 (the K-chunked scan path), explicit assignment, caller ids."""
    n, nq, dim, nlist = 1500, 24, 1024, 8
    rows = clustered(n + nq, dim, 6, 99)
    base, queries = rows[:n], rows[n:]
    cen = oracle.kmeans(base, nlist, seed=42, iters=2)
    assign = oracle.assign(base, cen)
    ocodec = oracle.Codec(dim, 2, 6)
    off, order, lists = oracle_lists(oracle, ocodec, base, cen, assign, True)
    user_ids = np.arange(n, dtype=np.int64) * 3 + 1000
    codec = uv.Codec(dim, 2, 6)
    ivf = uv.IvfIndex(codec, cen, centered=True)
    ivf.build(base, assign=assign, ids=user_ids)
    ex = ivf.export()
    assert np.array_equal(ex["ids"], user_ids[order])
    assert np.array_equal(ex["codes"], lists["codes"])
    gi, gs = ivf.search(queries, 10, 3)
    wi, ws = ocodec.ivf_search_topk(cen, off, user_ids[order], lists, True, queries, 3, 10)
    assert np.array_equal(gi, wi)
    assert bits_equal(gs, ws)


def test_rerank_bit_exact(oracle, uv):
    n, nq, dim, nlist = 3000, 32, 64, 16
    rows = clustered(n + nq, dim, 10, 3)
    base, queries = rows[:n], rows[n:]
    cen = oracle.kmeans(base, nlist, seed=42, iters=5)
    assign = oracle.assign(base, cen)
    ocodec = oracle.Codec(dim, 2, 6)
    off, ids, lists = oracle_lists(oracle, ocodec, base, cen, assign, False)
    ivf = uv.IvfIndex(uv.Codec(dim, 2, 6), cen)
    ivf.build(base)
    for k, rdepth, nprobe in [(10, 50, 4), (10, 10, 2), (5, 128, 16)]:
        gi, gs = ivf.search_with_rerank(queries, k, nprobe, rdepth, base)
        wi, ws = ocodec.ivf_search_rerank(cen, off, ids, lists, False, queries, nprobe, k,
                                          rdepth, base)
        assert np.array_equal(gi, wi)
        assert bits_equal(gs, ws)
    with pytest.raises(uv.UVError):
        ivf.search_with_rerank(queries, 10, 4, 50, base[:100])  # ids beyond db


def test_edge_cases(oracle, uv):
    dim, nlist = 64, 5
    rows = clustered(300, dim, 4, 11)
    cen = oracle.kmeans(rows, nlist, seed=42, iters=3)
    ivf = uv.IvfIndex(uv.Codec(dim, 2, 6), cen, centered=True)
    q = rows[:4].copy()
    q[1] = 0.0  # a zero query returns an empty result
    # empty index
    ids, sc = ivf.search(q, 5, 2)
    assert (ids == -1).all() and np.isneginf(sc).all()
    ivf.build(rows)
    ids, sc = ivf.search(q, 5, 0)  # nothing probed
    assert (ids == -1).all()
    ids, sc = ivf.search(q, 5, 9)  # nprobe > nlist: every list
    assert (ids[1] == -1).all()
    ocodec = oracle.Codec(dim, 2, 6)
    off, oids, lists = oracle_lists(oracle, ocodec, rows, cen, oracle.assign(rows, cen), True)
    wi, ws = ocodec.ivf_search_topk(cen, off, oids, lists, True, q, 9, 5)
    assert np.array_equal(ids, wi) and bits_equal(sc, ws)
    lists_out = ivf.probe(q, 7)
    assert (lists_out[:, 5:] == -1).all()
    with pytest.raises(uv.UVError):
        ivf.build(rows, assign=np.full(len(rows), nlist, np.uint32))  # list out of range


def test_device_tensors_in_and_out(oracle, uv):
    import torch

    dim, nlist = 64, 8
    rows = clustered(1000, dim, 5, 21)
    cen = oracle.kmeans(rows, nlist, seed=42, iters=5)
    got = uv.kmeans(torch.from_numpy(rows).cuda(), nlist, seed=42, iters=5)
    assert got.is_cuda and bits_equal(got.cpu().numpy(), cen)
    ivf = uv.IvfIndex(uv.Codec(dim, 2, 6), got, centered=False)
    ivf.build(torch.from_numpy(rows).cuda())
    qd = torch.from_numpy(rows[:16]).cuda()
    gi, gs = ivf.search(qd, 10, 3)
    hi, hs = ivf.search(rows[:16], 10, 3)
    assert gi.is_cuda and np.array_equal(gi.cpu().numpy(), hi) and bits_equal(gs.cpu().numpy(), hs)


@pytest.mark.parametrize("dim,nlist", [(128, 300), (256, 777), (2048, 512), (128, 1500)])
def test_tensor_core_probe_matches_oracle(oracle, uv, dim, nlist):
    """The probe from tensor-core dots plus exact rechecks (nlist >= 256)
    returns the oracle's lists: duplicated centroids (exact ties, lower list
    first), a zero centroid, zero and scaled queries, nprobe up to nlist; and
    the same lists and search results as the exact device probe."""
    rng = np.random.default_rng(dim + nlist)
    cen = clustered(nlist, dim, 8, dim + 5)
    cen[7] = cen[3]           # exact tie with list 3
    cen[nlist - 1] = cen[0]   # and with list 0
    cen[11] = 0.0             # cosine 0 against every query
    queries = clustered(60, dim, 8, dim + 6) * np.float32(3.0)
    queries[0] = 0.0          # every cosine 0: lists in index order
    queries[1] = cen[3] * np.float32(0.5)
    base = clustered(1500, dim, 8, dim + 7)
    codec = uv.Codec(dim, 2, 6)
    ivf = uv.IvfIndex(codec, cen, centered=False)
    ivf.build(base)
    try:
        for nprobe in (1, 4, 37, nlist):
            uv.set_tuning("ivf_tc_probe", 0)
            got = ivf.probe(queries, nprobe)
            if nprobe <= 37:
                want = np.stack([oracle.ivf_probe(cen, q, nprobe) for q in queries])
                assert np.array_equal(got, want), nprobe
            uv.set_tuning("ivf_tc_probe", 1)
            exact = ivf.probe(queries, nprobe)
            assert np.array_equal(got, exact), nprobe
            if nprobe in (1, 4):
                uv.set_tuning("ivf_tc_probe", 0)
                a = ivf.search(queries, 10, nprobe)
                uv.set_tuning("ivf_tc_probe", 1)
                b = ivf.search(queries, 10, nprobe)
                assert np.array_equal(a[0], b[0]) and bits_equal(a[1], b[1])
    finally:
        uv.set_tuning("ivf_tc_probe", 0)
