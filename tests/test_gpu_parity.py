"""GPU parity: the sm_100a library, called through its C ABI, against the CPU
oracle on the same seeded inputs.  Integer outputs (codes, start states,
windows, ids) must be identical; f32 outputs (rescale, rnorm, rotated rows,
scores) are compared bit for bit, since both sides perform the same IEEE
operations in the same order (the reference's own agreement bar,
1e-4 + 1e-4*|want| from simd.rs:278-322, is far looser)."""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest

from fixtures import rand_rows

pytestmark = pytest.mark.gpu
GOLD = Path(__file__).resolve().parent / "golden"


def _bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def _encode_both(uv, oracle, dim, bits, mem, rows, **kw):
    g = uv.Codec(dim, bits, mem, **{k: v for k, v in kw.items() if k != "centroids"})
    o = oracle.Codec(dim, bits, mem, **kw)
    cen = kw.get("centroids")
    got = g.encode(rows, centroids=cen)
    want = o.encode_batch(rows)
    return g, o, got, want


def _assert_records(got, want, cidx=False):
    np.testing.assert_array_equal(got["codes"], want["codes"])
    np.testing.assert_array_equal(got["start"], want["start"])
    np.testing.assert_array_equal(_bits(got["rescale"]), _bits(want["rescale"]))
    np.testing.assert_array_equal(_bits(got["rnorm"]), _bits(want["rnorm"]))
    if cidx:
        np.testing.assert_array_equal(got["cidx"], want["cidx"])


def test_code_table_and_signs_match(uv, oracle):
    for dim, bits, mem in [(128, 2, 8), (32, 2, 12), (1024, 4, 8), (96, 3, 7)]:
        g = uv.Codec(dim, bits, mem)
        o = oracle.Codec(dim, bits, mem)
        np.testing.assert_array_equal(g.code_table_bits(), _bits(o.table()))
        np.testing.assert_array_equal(g.rotation_sign_rounds(), o.signs())


@pytest.mark.parametrize("dim", [8, 32, 96, 128, 768, 1024, 2048])
def test_rotation_bit_exact(uv, oracle, dim):
    rows = rand_rows(64, dim, 3)
    g = uv.Codec(dim, 2, 4)
    o = oracle.Codec(dim, 2, 4)
    got = g.rotate(rows)
    want = np.stack([o.rotate(r) for r in rows])
    np.testing.assert_array_equal(_bits(got), _bits(want))


@pytest.mark.parametrize("dim,bits,mem,lam", [
    (128, 2, 6, 0.0), (128, 2, 8, 0.0), (96, 2, 10, 0.0), (256, 4, 6, 0.0),
    (128, 3, 7, 0.0), (128, 2, 8, 0.5),          # trellis.rs:2599-2629 shapes
    (32, 2, 12, 0.0),                            # smoke tier (M=12)
    (128, 2, 2, 0.0), (128, 2, 4, 0.0), (128, 2, 12, 0.0),  # memory sweep
    (128, 1, 8, 0.0), (128, 4, 8, 0.0), (64, 1, 3, 0.0), (64, 1, 1, 0.0),
])
def test_encode_bit_exact(uv, oracle, dim, bits, mem, lam):
    rows = oracle.rand_unit(300, dim, 4242 + mem)
    _, _, got, want = _encode_both(uv, oracle, dim, bits, mem, rows, branch_lambda=lam)
    _assert_records(got, want)


@pytest.mark.parametrize("dim,bits", [(1024, 1), (1024, 2), (1024, 4), (2048, 2)])
def test_encode_wide_rows_bit_exact(uv, oracle, dim, bits):
    """d=1024/2048 keep back-pointers in global scratch (chunked traceback)."""
    rows = rand_rows(96, dim, 7 + bits)
    _, _, got, want = _encode_both(uv, oracle, dim, bits, 8, rows)
    _assert_records(got, want)


@pytest.mark.parametrize("dim,bits,mem,n,kw", [
    (128, 3, 12, 40, {}),                       # window 15 at 3 bits: staged
    (128, 4, 12, 24, {}),                       # window 16 at 4 bits: staged
    (64, 3, 14, 16, {}),                        # window 17
    (64, 4, 14, 12, {}),                        # window 18
    (32, 3, 16, 6, {}),                         # window 19: the 3-bit M = 16 cell
    (32, 4, 16, 4, {}),                         # window 20: the 4-bit M = 16 cell
    (64, 3, 13, 16, {"branch_lambda": 0.5, "start_bits": 9}),
    (64, 2, 1, 200, {}),                        # mem < bits: the general pass
    (64, 3, 1, 200, {}),
    (64, 4, 2, 200, {"branch_lambda": 0.5}),
    (96, 4, 3, 200, {"start_bits": 2}),
])
def test_encode_staged_bit_exact(uv, oracle, dim, bits, mem, n, kw):
    """The shapes the resident encoders do not hold (encode_staged.cu):
    windows of 15 and more bits at 3 and 4 bits per coordinate, and the
    reference's general Viterbi pass for mem < bits (src/trellis.rs:1348-1387)."""
    rows = oracle.rand_unit(n, dim, 700 + mem * 7 + bits)
    _, _, got, want = _encode_both(uv, oracle, dim, bits, mem, rows, **kw)
    _assert_records(got, want)


def test_encode_staged_centered_raw_rows_and_search(uv, oracle):
    """Centering, non-unit rows and a search over staged records (a 2^15
    entry code table, read through L1 by the scan kernels)."""
    rows = rand_rows(600, 128, 41) * np.float32(5.0)
    cen = oracle.kmeans(rows, 3, 42)
    _, _, got, want = _encode_both(uv, oracle, 128, 3, 12, rows, centroids=cen)
    _assert_records(got, want, cidx=True)
    qs = rand_rows(20, 128, 42)
    g, ix = _index(uv, 128, 3, 12, rows)
    o = oracle.Codec(128, 3, 12)
    enc = o.encode_batch(rows)
    for k in (10, 100, 600):
        ids, scores = ix.search(qs, k, mips=True)
        wids, wscores = o.search_topk(enc, qs, k, norms=oracle.l2_norms(rows))
        np.testing.assert_array_equal(ids, wids)
        np.testing.assert_array_equal(_bits(scores), _bits(wscores))


@pytest.mark.parametrize("dim,bits,mem,n,kw", [
    (128, 2, 13, 48, {}),                       # 2 CTAs per row
    (128, 2, 14, 40, {"branch_lambda": 0.5}),   # 4 CTAs, anisotropic metric
    (64, 1, 14, 40, {"start_bits": 9}),         # 2 CTAs, restricted free start
    (64, 2, 16, 24, {}),                        # 16 CTAs (8192 threads per row)
    (32, 1, 17, 24, {}),                        # 16 CTAs at b = 1
])
def test_encode_cluster_bit_exact(uv, oracle, dim, bits, mem, n, kw):
    """mem + bits >= 15: one thread-block cluster per row (encode_cluster.cu),
    costs exchanged through distributed shared memory."""
    rows = oracle.rand_unit(n, dim, 900 + mem + bits)
    _, _, got, want = _encode_both(uv, oracle, dim, bits, mem, rows, **kw)
    _assert_records(got, want)


def test_encode_cluster_centered_and_raw_rows(uv, oracle):
    rows = rand_rows(32, 128, 31) * np.float32(7.0)
    cen = oracle.kmeans(rows, 4, 42)
    _, _, got, want = _encode_both(uv, oracle, 128, 2, 13, rows, centroids=cen)
    _assert_records(got, want, cidx=True)


def test_encode_raw_heavy_tailed_rows(uv, oracle):
    """Non-unit, non-negative integer rows (the flat-scan corpus shape)."""
    rng = np.random.default_rng(5)
    x = np.where(rng.random((500, 128)) < 0.4, 0,
                 np.minimum(255, 1 + rng.geometric(1 / 20, (500, 128)))).astype(np.float32)
    x -= x.mean(0, dtype=np.float64).astype(np.float32)
    _, _, got, want = _encode_both(uv, oracle, 128, 2, 8, x)
    _assert_records(got, want)


def test_encode_centered_bit_exact(uv, oracle):
    """with_centroids (src/trellis.rs:952-956): assignment, unit residual, rnorm."""
    rows = oracle.rand_unit(400, 128, 77)
    cen = oracle.kmeans(rows, 8, 42)
    _, _, got, want = _encode_both(uv, oracle, 128, 2, 8, rows, centroids=cen)
    _assert_records(got, want, cidx=True)
    mean = rows.mean(0).astype(np.float32)[None, :]
    _, _, got, want = _encode_both(uv, oracle, 128, 2, 8, rows, centroids=mean)
    _assert_records(got, want, cidx=True)


def test_encode_degenerate_rows(uv, oracle):
    """NaN, one-NaN, zero and +inf rows (src/trellis.rs:2360-2385)."""
    dim = 64
    rows = list(oracle.rand_unit(2, dim, 7))
    rows.append(np.full(dim, np.nan, np.float32))
    one = rows[0].copy()
    one[3] = np.nan
    rows.append(one)
    rows.append(np.zeros(dim, np.float32))
    rows.append(np.full(dim, np.inf, np.float32))
    rows.append(np.full(dim, 1e30, np.float32))
    rows = np.stack(rows).astype(np.float32)
    _, _, got, want = _encode_both(uv, oracle, dim, 2, 6, rows)
    np.testing.assert_array_equal(got["codes"], want["codes"])
    np.testing.assert_array_equal(got["start"], want["start"])
    assert (got["start"] < 64).all()


def test_encode_rotated_matches(uv, oracle):
    g = uv.Codec(128, 3, 6)
    o = oracle.Codec(128, 3, 6)
    rows = oracle.rand_unit(64, 128, 9)
    u_r = np.stack([o.rotate(r / np.float32(max(oracle.l2_norm(r), 1.1920929e-07))) for r in rows])
    codes, start = g.encode_rotated(u_r)
    for i in range(64):
        wc, ws = o.encode_rotated(u_r[i])
        assert bytes(codes[i]) == bytes(wc) and int(start[i]) == ws


@pytest.mark.parametrize("dim,bits,mem", [(128, 2, 12), (128, 3, 12), (128, 4, 12), (64, 1, 8),
                                          (64, 4, 14), (32, 1, 16)])
def test_windows_match_oracle(uv, oracle, dim, bits, mem):
    """trellis.rs:2915-2952 window widths 10..18 bits."""
    o = oracle.Codec(dim, bits, mem)
    rows = oracle.rand_unit(8, dim, 31 + mem)
    enc = o.encode_batch(rows)
    g = uv.Codec(dim, bits, mem)
    got = g.windows(enc["codes"], enc["start"])
    want = np.stack([o.windows(enc["codes"][i], int(enc["start"][i])) for i in range(8)])
    np.testing.assert_array_equal(got, want)


def test_decode_and_digest_match(uv, oracle):
    o = oracle.Codec(128, 2, 8)
    g = uv.Codec(128, 2, 8)
    enc = o.encode_batch(oracle.rand_unit(50, 128, 3))
    got = g.decode(enc["codes"], enc["start"])
    want = np.stack([o.decode_codes(enc["codes"][i], int(enc["start"][i])) for i in range(50)])
    np.testing.assert_array_equal(_bits(got), _bits(want))
    assert g.digest(enc["codes"], enc["start"]) == oracle.digest(enc["codes"], enc["start"])


def _index(uv, dim, bits, mem, rows, centroids=None):
    g = uv.Codec(dim, bits, mem)
    ix = uv.Index(g)
    if centroids is not None:
        ix.set_centroids(centroids)
    ix.add_batch(rows)
    return g, ix


@pytest.mark.parametrize("mips", [True, False])
def test_flat_search_matches_oracle(uv, oracle, mips):
    """Config 1 shape: 10k x 128 N(0,1), M=8, 2 bits, 100 queries, top-10/100."""
    rows = rand_rows(10_000, 128, 0)
    qs = rand_rows(100, 128, 1)
    g, ix = _index(uv, 128, 2, 8, rows)
    o = oracle.Codec(128, 2, 8)
    enc = o.encode_batch(rows)
    ex = ix.export()
    np.testing.assert_array_equal(ex["codes"], enc["codes"])
    norms = oracle.l2_norms(rows) if mips else None
    if mips:
        np.testing.assert_array_equal(_bits(ex["norms"]), _bits(norms))
    for k in (10, 100):
        ids, scores = ix.search(qs, k, mips=mips)
        wids, wscores = o.search_topk(enc, qs, k, norms=norms)
        np.testing.assert_array_equal(ids, wids)
        np.testing.assert_array_equal(_bits(scores), _bits(wscores))


@pytest.mark.parametrize("dim,bits,mem", [(32, 2, 12), (64, 1, 8), (96, 3, 7), (256, 4, 6),
                                          (384, 2, 8), (128, 2, 4), (16, 1, 12),
                                          (80, 2, 8), (48, 3, 6)])
def test_flat_search_shapes(uv, oracle, dim, bits, mem):
    rows = rand_rows(777, dim, dim)
    qs = rand_rows(45, dim, dim + 1)
    g, ix = _index(uv, dim, bits, mem, rows)
    o = oracle.Codec(dim, bits, mem)
    enc = o.encode_batch(rows)
    ids, scores = ix.search(qs, 17, mips=True)
    wids, wscores = o.search_topk(enc, qs, 17, norms=oracle.l2_norms(rows))
    np.testing.assert_array_equal(ids, wids)
    np.testing.assert_array_equal(_bits(scores), _bits(wscores))


def test_flat_search_centered(uv, oracle):
    rows = oracle.rand_unit(600, 128, 11)
    qs = oracle.rand_unit(40, 128, 12)
    cen = oracle.kmeans(rows, 4, 42)
    g, ix = _index(uv, 128, 2, 8, rows, centroids=cen)
    o = oracle.Codec(128, 2, 8, centroids=cen)
    enc = o.encode_batch(rows)
    ids, scores = ix.search(qs, 10)
    wids, wscores = o.search_topk(enc, qs, 10)
    np.testing.assert_array_equal(ids, wids)
    np.testing.assert_array_equal(_bits(scores), _bits(wscores))


def test_search_edge_cases(uv, oracle):
    dim = 128
    rows = rand_rows(45, dim, 2)
    rows[7] = rows[3]  # duplicate record: exact tie, broken by id
    rows[20] = 0.0     # zero row: rescale = +inf, score 0
    qs = rand_rows(5, dim, 4)
    qs[1] = 0.0        # degenerate query: no results
    g, ix = _index(uv, dim, 2, 8, rows)
    o = oracle.Codec(dim, 2, 8)
    enc = o.encode_batch(rows)
    ids, scores = ix.search(qs, 64)   # k > N
    wids, wscores = o.search_topk(enc, qs, 64)
    np.testing.assert_array_equal(ids, wids)
    np.testing.assert_array_equal(_bits(scores), _bits(wscores))
    assert (ids[1] == -1).all() and (ids[0, 45:] == -1).all()
    # empty index
    e = uv.Index(g)
    ids, _ = e.search(qs, 5)
    assert (ids == -1).all()


def test_smoke_bundle_through_the_gpu(uv, oracle):
    """The reference's retained smoke run reproduced end to end on the GPU."""
    base = np.fromfile(GOLD / "smoke_base.f32", "<f4").reshape(128, 32)
    query = np.fromfile(GOLD / "smoke_query.f32", "<f4").reshape(16, 32)
    exp = json.loads((GOLD / "smoke_expected.json").read_text())
    g, ix = _index(uv, 32, 2, 12, base)
    ids, _ = ix.search(query, 100)
    gold = oracle.exact_topk(base, query, 100, cosine=True)
    got = np.array([[len(set(gold[q, :k]) & set(ids[q, :k])) / k for k in (1, 10, 100)]
                    for q in range(16)])
    np.testing.assert_array_equal(got, np.array(exp["per_query_recall_1_10_100"]))


def test_topk_merge(uv):
    rng = np.random.default_rng(0)
    nq, L, k = 7, 5, 12
    scores = rng.integers(0, 6, (nq, L, k)).astype(np.float32)  # many ties
    ids = rng.permutation(nq * L * k).reshape(nq, L, k).astype(np.int64)
    ids[0, 1, 3:] = -1
    order = np.lexsort((ids, -scores), axis=-1)
    scores = np.take_along_axis(scores, order, -1)
    ids = np.take_along_axis(ids, order, -1)
    got_ids, got_scores = uv.topk_merge(ids, scores, 9)
    for q in range(nq):
        cand = [(-s, i) for s, i in zip(scores[q].ravel(), ids[q].ravel()) if i >= 0]
        cand.sort()
        want = [i for _, i in cand[:9]]
        assert list(got_ids[q]) == want


def test_device_tensors_round_trip(uv, oracle):
    """Device-resident inputs/outputs (torch CUDA) give the same records."""
    import torch

    rows = rand_rows(256, 128, 9)
    g = uv.Codec(128, 2, 8)
    host = g.encode(rows)
    dev = g.encode(torch.from_numpy(rows).cuda())
    torch.cuda.synchronize()
    np.testing.assert_array_equal(dev["codes"].cpu().numpy(), host["codes"])
    np.testing.assert_array_equal(dev["start"].cpu().numpy().view(np.uint32), host["start"])
    ix = uv.Index(g)
    ix.add_batch(torch.from_numpy(rows).cuda())
    qs = torch.from_numpy(rand_rows(8, 128, 10)).cuda()
    ids, _ = ix.search(qs, 10, mips=True)
    torch.cuda.synchronize()
    ids_h, _ = ix.search(qs.cpu().numpy(), 10, mips=True)
    np.testing.assert_array_equal(ids.cpu().numpy(), ids_h)


@pytest.mark.parametrize("dim,bits,k", [(1024, 2, 10), (1024, 1, 100), (1024, 4, 17),
                                        (2048, 2, 10), (400, 3, 33)])
def test_flat_search_wide_rows(uv, oracle, dim, bits, k):
    """Rows wider than 384 take the K-chunked scan (128-coordinate chunks)."""
    rows = rand_rows(1500, dim, dim + bits)
    qs = rand_rows(70, dim, dim + bits + 1)
    g, ix = _index(uv, dim, bits, 8, rows)
    o = oracle.Codec(dim, bits, 8)
    enc = o.encode_batch(rows)
    for mips in (True, False):
        ids, scores = ix.search(qs, k, mips=mips)
        wids, wscores = o.search_topk(enc, qs, k, norms=oracle.l2_norms(rows) if mips else None)
        np.testing.assert_array_equal(ids, wids)
        np.testing.assert_array_equal(_bits(scores), _bits(wscores))
