"""The flat search of a base split into shards (uv_index_search_begin /
uv_search_set_bounds / uv_search_finish, uv_topk_pack, uv_topk_merge_packed),
on one GPU: every shard is its own index on cuda:0 and the collectives of
the multi-GPU protocol are emulated by concatenation and slicing (the same
layouts NCCL's all-gather and all-to-all produce).  The merged answer must
be the unsharded index's and the oracle's, ids and score bits."""
from __future__ import annotations

import numpy as np
import pytest

from fixtures import rand_rows

pytestmark = pytest.mark.gpu


def _bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def _shards(uv, rows, n_shards, dim=128, bits=2, mem=8, centroids=None):
    codec = uv.Codec(dim, bits, mem)
    out = []
    for r in range(n_shards):
        lo, hi = r * len(rows) // n_shards, (r + 1) * len(rows) // n_shards
        ix = uv.Index(codec)
        if centroids is not None:
            ix.set_centroids(centroids)
        ix.add(np.arange(lo, hi, dtype=np.int64), rows[lo:hi])
        out.append(ix)
    return codec, out


def _protocol(uv, shards, qs, k, mips, share=True, deferred=False):
    import torch

    n = len(shards)
    if deferred:  # device queries: the deferred finish takes device buffers
        qs = torch.from_numpy(np.ascontiguousarray(qs)).cuda()
    # without sharing, each shard searches as a base of its own (n_shards 1)
    ss = [ix.search_begin(qs, k, mips=mips, n_shards=n if share else 1) for ix in shards]
    if share:
        gathered = torch.cat([torch.as_tensor(s.bounds).cuda() for s in ss], 0)
        for s in ss:
            s.set_bounds(gathered, n)
    res = [s.finish(deferred=deferred) for s in ss]
    if deferred:
        assert not any(s.check() for s in ss)  # no overflow on these inputs
    for s in ss:
        s.close()
    packed = [uv.topk_pack(torch.as_tensor(i).cuda(), torch.as_tensor(sc).cuda())
              for i, sc in res]
    nq = len(qs)
    out_i, out_s = [], []
    for r in range(n):
        lo, hi = r * nq // n, (r + 1) * nq // n
        rows = hi - lo
        recv = torch.cat([p[lo:hi].reshape(-1) for p in packed])
        i, sc = uv.topk_merge_packed(recv, rows, n, k, k, row_stride=k, list_stride=rows * k)
        out_i.append(i.cpu().numpy())
        out_s.append(sc.cpu().numpy())
    return np.concatenate(out_i), np.concatenate(out_s)


@pytest.mark.parametrize("n_shards,k,mips", [(2, 100, True), (4, 100, True), (4, 10, False),
                                             (3, 17, True), (5, 128, False)])
def test_sharded_search_equals_one_index(uv, oracle, n_shards, k, mips):
    rows = rand_rows(60_000, 128, 70 + n_shards)
    rows[123] = rows[59_000]  # an exact tie across shards, broken by id
    qs = rand_rows(301, 128, 80 + n_shards)
    codec, shards = _shards(uv, rows, n_shards)
    ids, scores = _protocol(uv, shards, qs, k, mips)
    one = uv.Index(codec)
    one.add_batch(rows)
    wids, wsc = one.search(qs, k, mips=mips)
    np.testing.assert_array_equal(ids, wids)
    np.testing.assert_array_equal(_bits(scores), _bits(wsc))
    o = oracle.Codec(128, 2, 8)
    ex = one.export()  # the GPU's records (their bit-exactness is tested elsewhere)
    rec = {"codes": ex["codes"], "start": ex["start"], "rescale": ex["rescale"]}
    oids, osc = o.search_topk(rec, qs[:40], k, norms=ex["norms"] if mips else None)
    np.testing.assert_array_equal(ids[:40], oids)
    np.testing.assert_array_equal(_bits(scores[:40]), _bits(osc))
    # without the shared threshold every shard keeps its own top k: same answer
    ids2, scores2 = _protocol(uv, shards, qs, k, mips, share=False)
    np.testing.assert_array_equal(ids2, wids)
    # the deferred finish (work queued, outcome checked after the merge)
    ids3, scores3 = _protocol(uv, shards, qs, k, mips, deferred=True)
    np.testing.assert_array_equal(ids3, wids)
    np.testing.assert_array_equal(_bits(scores3), _bits(wsc))


def test_shared_threshold_prunes_candidates(uv):
    """The shards score exactly fewer candidates with the shared bound."""
    import torch

    # shards large enough that each alone also runs the prefilter
    rows = rand_rows(800_000, 128, 91)
    qs = rand_rows(256, 128, 92)
    _, shards = _shards(uv, rows, 4)
    counts = {}
    for share in (False, True):
        s_all = [x.search_begin(qs, 100, mips=True, n_shards=4 if share else 1) for x in shards]
        if share:
            g = torch.cat([torch.as_tensor(s.bounds).cuda() for s in s_all], 0)
            for s in s_all:
                s.set_bounds(g, 4)
        total = 0
        for s in s_all:
            s.finish()
            total += uv.profile_read("tc_candidates")[1]
            s.close()
        counts[share] = total
    assert counts[True] < counts[False]
    # with several shards the shared threshold is required before finish
    s = shards[0].search_begin(qs, 100, mips=True, n_shards=4)
    assert s.bounds.shape == (256, 50)  # min(k, 2 * ceil(k / 4)) per query
    with pytest.raises(uv.UVError):
        s.finish()
    s.close()


def test_sharded_search_other_paths(uv, oracle):
    """Shards on the exact path (centered index), the full ranking (k above
    128), host queries and outputs, an empty shard and uneven query slices."""
    rows = oracle.rand_unit(3000, 128, 93)
    qs = oracle.rand_unit(13, 128, 94)
    cen = oracle.kmeans(rows, 4, 42)
    codec, shards = _shards(uv, rows, 3, centroids=cen)
    one = uv.Index(codec)
    one.set_centroids(cen)
    one.add_batch(rows)
    for k in (10, 300):
        ids, scores = _protocol(uv, shards, qs, k, False)
        wids, wsc = one.search(qs, k)
        np.testing.assert_array_equal(ids, wids)
        np.testing.assert_array_equal(_bits(scores), _bits(wsc))
    # an empty shard takes part like the others
    codec2, shards2 = _shards(uv, rows[:2000], 2)
    empty = uv.Index(codec2)
    ids, scores = _protocol(uv, shards2 + [empty], qs, 10, True)
    one2 = uv.Index(codec2)
    one2.add_batch(rows[:2000])
    wids, wsc = one2.search(qs, 10, mips=True)
    np.testing.assert_array_equal(ids, wids)
    np.testing.assert_array_equal(_bits(scores), _bits(wsc))


def test_merge_packed_large_rows(uv):
    """Above 8192 entries per row the packed merge sorts: 8 lists of 1500."""
    import torch

    rng = np.random.default_rng(3)
    nq, L, kin, k = 5, 8, 1500, 2000
    sc = np.sort(rng.integers(0, 50, (nq, L, kin)).astype(np.float32), axis=2)[..., ::-1]
    ids = rng.permutation(nq * L * kin).reshape(nq, L, kin).astype(np.int64)
    order = np.lexsort((ids, -sc), axis=-1)
    sc = np.ascontiguousarray(np.take_along_axis(sc, order, -1))
    ids = np.ascontiguousarray(np.take_along_axis(ids, order, -1))
    ids[1, 2, 700:] = -1
    sc[1, 2, 700:] = -np.inf
    packed = uv.topk_pack(torch.from_numpy(ids).cuda(), torch.from_numpy(sc).cuda())
    got_i, got_s = uv.topk_merge_packed(packed, nq, L, kin, k)
    want_i, want_s = uv.topk_merge(ids, sc, k)
    np.testing.assert_array_equal(got_i.cpu().numpy(), want_i)
    for q in range(nq):
        cand = sorted((-s, i) for s, i in zip(sc[q].ravel(), ids[q].ravel()) if i >= 0)
        assert list(want_i[q]) == [i for _, i in cand[:k]]


@pytest.mark.parametrize("L,kin,k", [(8, 100, 100), (5, 12, 9), (4, 200, 150), (16, 64, 40)])
def test_merge_sorted_and_unsorted_lists(uv, L, kin, k):
    """The k-way merge (one warp per row below 512 entries, one CTA above)
    against a host reference, with exact ties, unfilled tails and a row
    whose lists are not sorted by (score, id) (the bitonic fallback)."""
    rng = np.random.default_rng(L * 1000 + kin)
    nq = 7
    sc = rng.integers(0, 40, (nq, L, kin)).astype(np.float32)
    ids = rng.permutation(nq * L * kin).reshape(nq, L, kin).astype(np.int64)
    order = np.lexsort((ids, -sc), axis=-1)
    sc = np.ascontiguousarray(np.take_along_axis(sc, order, -1))
    ids = np.ascontiguousarray(np.take_along_axis(ids, order, -1))
    ids[2, 1, kin // 3:] = -1
    sc[2, 1, kin // 3:] = -np.inf
    ids[4, 0, :2] = ids[4, 0, 1::-1].copy()  # ids out of order at a tie or not
    sc[4, 0, :2] = 50.0
    got_i, got_s = uv.topk_merge(ids, sc, k)
    for q in range(nq):
        cand = sorted((-s, i) for s, i in zip(sc[q].ravel(), ids[q].ravel()) if i >= 0)
        want = [i for _, i in cand[:k]] + [-1] * max(0, k - len(cand))
        assert list(got_i[q]) == want, q
        assert list(got_s[q][:len(cand)]) == [-s for s, _ in cand[:k]][:len(cand)]


@pytest.mark.parametrize("n_shards,nprobe,tc", [(3, 4, 0), (4, 16, 2), (2, 1, 1)])
def test_ivf_sharded_by_lists_with_a_split_probe(oracle, uv, n_shards, nprobe, tc):
    """An IVF base dealt to shards by posting list (shard.ivf_list_owners):
    shard r probes only its query slice, the lists are concatenated (the
    all-gather's layout), every shard scans the probed lists it holds
    (search_lists; the others are empty here and skipped), the packed lists
    merge per query slice -- equal to the unsharded IVF search, with the
    tensor-core and the CUDA-core list scans."""
    import torch

    from ultravec_ann_b200.shard import ivf_list_owners, ivf_owned_rows

    rng = np.random.default_rng(n_shards * 10 + nprobe)
    dim, nlist, n, nq, k = 256, 24, 6000, 37, 10
    c = rng.standard_normal((8, dim)).astype(np.float32)
    base = c[rng.integers(0, 8, n)] + np.float32(0.5) * rng.standard_normal((n, dim)).astype(
        np.float32)
    qs = base[rng.integers(0, n, nq)] + np.float32(0.1) * rng.standard_normal((nq, dim)).astype(
        np.float32)
    cen = oracle.kmeans(base, nlist, seed=42, iters=2)
    asg = oracle.assign(base, cen)
    codec = uv.Codec(dim, 2, 8)
    whole = uv.IvfIndex(codec, cen, centered=True)
    whole.build(base, assign=asg)
    owners = ivf_list_owners(np.bincount(asg, minlength=nlist), n_shards)
    shards = []
    for r in range(n_shards):
        rows = ivf_owned_rows(asg, owners, r)
        ix = uv.IvfIndex(codec, cen, centered=True)
        ix.build(base[rows], assign=asg[rows], ids=rows.astype(np.int64))
        shards.append(ix)
    uv.set_tuning("ivf_tc", tc)
    try:
        want_i, want_s = whole.search(qs, k, nprobe)
        lists = np.concatenate([shards[r].probe(qs[r * nq // n_shards:(r + 1) * nq // n_shards],
                                                nprobe) for r in range(n_shards)])
        assert np.array_equal(lists, whole.probe(qs, nprobe))
        res = [ix.search_lists(qs, k, lists) for ix in shards]
    finally:
        uv.set_tuning("ivf_tc", 0)
    packed = [uv.topk_pack(torch.as_tensor(i).cuda(), torch.as_tensor(s).cuda()) for i, s in res]
    out_i, out_s = [], []
    for r in range(n_shards):
        lo, hi = r * nq // n_shards, (r + 1) * nq // n_shards
        rows = hi - lo
        recv = torch.cat([p[lo:hi].reshape(-1) for p in packed])
        i, s = uv.topk_merge_packed(recv, rows, n_shards, k, k, row_stride=k,
                                    list_stride=rows * k)
        out_i.append(i.cpu().numpy())
        out_s.append(s.cpu().numpy())
    got_i, got_s = np.concatenate(out_i), np.concatenate(out_s)
    assert np.array_equal(got_i, want_i)
    assert np.array_equal(_bits(got_s), _bits(want_s))
    # a list id past nlist is refused
    bad = lists.copy()
    bad[0, 0] = nlist
    with pytest.raises(uv.UVError):
        shards[0].search_lists(qs, k, bad)
