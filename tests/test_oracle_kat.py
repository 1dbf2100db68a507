"""Pins the CPU oracle to the reference.

The reference ships no golden code bytes, so the oracle is pinned two ways:
  * its retained smoke run (results/generated/smoke-synthetic): per-query
    Recall@1/10/100 and reconstruction MSE of the 2-bit M=12 trellis over a
    numpy-generated corpus, reproduced here exactly;
  * ports of the reference's own known-answer and consistency tests
    (trellis.rs, lib.rs, simd.rs, ivf.rs), each cited.
"""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest

GOLD = Path(__file__).resolve().parent / "golden"
EPS = np.float32(1.1920929e-07)


def _smoke():
    base = np.fromfile(GOLD / "smoke_base.f32", "<f4").reshape(128, 32)
    query = np.fromfile(GOLD / "smoke_query.f32", "<f4").reshape(16, 32)
    exp = json.loads((GOLD / "smoke_expected.json").read_text())
    return base, query, exp


def test_smoke_bundle_recall_per_query(oracle):
    """results/generated/smoke-synthetic: trellis rows of per-query.csv."""
    base, query, exp = _smoke()
    c = oracle.Codec(32, 2, 12)
    idx = c.encode_batch(base)
    ids, _ = c.search_topk(idx, query, 100)
    gold = oracle.exact_topk(base, query, 100, cosine=True)
    got = np.array([[len(set(gold[q, :k]) & set(ids[q, :k])) / k for k in (1, 10, 100)]
                    for q in range(16)])
    np.testing.assert_array_equal(got, np.array(exp["per_query_recall_1_10_100"]))
    np.testing.assert_allclose(got.mean(0), exp["mean_recall_1_10_100"], atol=5e-4)


def test_smoke_bundle_reconstruction_mse(oracle):
    """stdout.txt trellis row: recon MSE 0.04712 (lib.rs:159-187 protocol)."""
    base, _, exp = _smoke()
    c = oracle.Codec(32, 2, 12)
    idx = c.encode_batch(base)
    tot = 0.0
    for i in range(base.shape[0]):
        x = base[i]
        nx = np.float32(max(oracle.l2_norm(x), EPS))
        r = c.reconstruct_unit(idx["codes"][i], int(idx["start"][i]))
        d = (x / nx - r).astype(np.float64)
        tot += float((d * d).sum())
    assert f"{tot / base.shape[0]:.5f}" == exp["recon_mse"]


@pytest.mark.parametrize("dim,bits,mem,lam", [(128, 2, 6, 0.0), (128, 2, 8, 0.0),
                                              (96, 2, 10, 0.0), (256, 4, 6, 0.0),
                                              (128, 3, 7, 0.0), (128, 2, 8, 0.5)])
def test_fast_viterbi_is_byte_identical_to_triple_loop(oracle, dim, bits, mem, lam):
    """trellis.rs:2599-2629 simd_v1_encode_is_byte_identical_to_scalar."""
    c = oracle.Codec(dim, bits, mem, branch_lambda=lam)
    rows = oracle.rand_unit(40, dim, 4242 + mem)
    for v in rows:
        codes, start, *_ = c.encode(v)
        rc, rs = c.encode_scalar_ref(v)
        assert bytes(codes) == bytes(rc)
        assert start == rs


@pytest.mark.parametrize("n_states,n_emit", [(8, 2), (8, 4), (16, 4), (32, 16), (64, 8)])
def test_acs_tie_break_on_deliberate_ties(oracle, n_states, n_emit):
    """trellis.rs:2542-2597: integer-valued cost s%3 and metric w%5 make ties
    abundant; ascending k with strict `<` must win them."""
    b = n_emit.bit_length() - 1
    cost = np.array([s % 3 for s in range(n_states)], np.float32)
    total = np.array([w % 5 for w in range(n_states * n_emit)], np.float32)
    want_next = np.zeros(n_states, np.float32)
    want_back = np.zeros(n_states, np.uint8)
    for ns in range(n_states):
        best, bk = cost[ns >> b] + total[ns], 0
        for k in range(1, n_emit):
            w = ns + k * n_states
            cand = cost[w >> b] + total[w]
            if cand < best:
                best, bk = cand, k
        want_next[ns], want_back[ns] = best, bk
    nxt, back = oracle.acs_step(cost, total, n_states, n_emit)
    np.testing.assert_array_equal(back, want_back)
    np.testing.assert_array_equal(nxt, want_next)


def _chain(c, codes, start):
    em = oracle_unpack(codes, c.bits, c.dim)
    out, state = [], start
    mask = (1 << c.mem) - 1
    for e in em:
        w = (state << c.bits) | int(e)
        out.append(w)
        state = w & mask
    return np.array(out, np.uint32)


def oracle_unpack(codes, bits, n):
    import oracle as O

    return O.unpack_indices(codes, bits, n)


@pytest.mark.parametrize("dim,bits,mem", [(128, 2, 12), (128, 3, 12), (128, 4, 12), (64, 1, 8),
                                          (64, 4, 14), (32, 1, 16)])
def test_windows_match_the_state_chain(oracle, dim, bits, mem):
    """trellis.rs:2915-2952 (15/16/17/18-bit windows, bits not dividing 8)."""
    c = oracle.Codec(dim, bits, mem)
    for v in oracle.rand_unit(8, dim, 31 + mem):
        codes, start, *_ = c.encode(v)
        np.testing.assert_array_equal(c.windows(codes, start), _chain(c, codes, start))


@pytest.mark.parametrize("dim,bits,mem", [(64, 2, 6), (128, 3, 6), (128, 2, 10), (128, 1, 12)])
def test_window_at_matches_the_state_chain(oracle, dim, bits, mem):
    """trellis.rs:2304-2324."""
    c = oracle.Codec(dim, bits, mem)
    for v in oracle.rand_unit(4, dim, 5):
        codes, start, *_ = c.encode(v)
        chain = _chain(c, codes, start)
        for i in range(dim):
            assert c.window_at(codes, start, i) == chain[i]


def test_encode_rotated_reproduces_encode_codes(oracle):
    """trellis.rs:2329-2339."""
    c = oracle.Codec(128, 3, 6)
    for row in oracle.rand_unit(16, 128, 9):
        unit = row / np.float32(max(oracle.l2_norm(row), EPS))
        codes_a, start_a = c.encode_rotated(c.rotate(unit.astype(np.float32)))
        codes_b, start_b, *_ = c.encode(row)
        assert bytes(codes_a) == bytes(codes_b) and start_a == start_b


def test_decode_codes_normalized_is_reconstruct_unit(oracle):
    """trellis.rs:2343-2356."""
    c = oracle.Codec(128, 2, 8)
    for row in oracle.rand_unit(8, 128, 3):
        codes, start, *_ = c.encode(row)
        raw = c.decode_codes(codes, start)
        unit = raw / np.float32(oracle.l2_norm(raw))
        np.testing.assert_allclose(unit, c.reconstruct_unit(codes, start), atol=1e-6)


def test_degenerate_rows_give_valid_records(oracle):
    """trellis.rs:2360-2385 (exact encoder): NaN, one-NaN, zero, +inf rows."""
    dim = 64
    rows = list(oracle.rand_unit(2, dim, 7))
    rows.append(np.full(dim, np.nan, np.float32))
    one = rows[0].copy()
    one[3] = np.nan
    rows.append(one)
    rows.append(np.zeros(dim, np.float32))
    rows.append(np.full(dim, np.inf, np.float32))
    c = oracle.Codec(dim, 2, 6)
    for row in rows:
        codes, start, rescale, *_ = c.encode(row)
        assert len(codes) == dim * 2 // 8
        assert 0 <= start < (1 << 6)


def test_record_bytes_follow_the_scalar_widths(oracle):
    """trellis.rs:2864-2913: payload = ceil(dim*bits/8), start = ceil(M/8)."""
    for dim, bits in [(128, 2), (1024, 1), (1024, 4), (2048, 2), (96, 3)]:
        assert oracle.Codec(dim, bits, 8).code_bytes == (dim * bits + 7) // 8


def test_computed_code_is_approximately_gaussian(oracle):
    """trellis.rs:2415-2433 at the reference default (M=12, 2 bits)."""
    t = oracle.Codec(64, 2, 12).table().astype(np.float32)
    n = np.float32(len(t))
    mean = np.float32(0)
    for v in t:
        mean += v
    mean /= n
    var = np.float32(0)
    for v in t:
        var += (v - mean) * (v - mean)
    var /= n
    assert abs(mean) < 1e-4 and abs(var - 1) < 1e-3
    maxv = float(np.abs(t).max())
    ext = float(np.sqrt(2 * np.log(n)))
    assert 0.5 * ext < maxv < 2 * ext


def _xorshift_stream(seed, n):
    """simd.rs:268-276 fixture generator (xorshift64*)."""
    st = seed
    out = []
    m = (1 << 64) - 1
    for _ in range(n):
        st ^= st >> 12
        st ^= (st << 25) & m
        st ^= st >> 27
        v = ((st * 0x2545F4914F6CDD1D) & m) >> 11
        out.append(np.float32((np.float32(v / float(1 << 53)) - np.float32(0.5)) * np.float32(4.0)))
    return np.array(out, np.float32)


@pytest.mark.parametrize("n", [1, 7, 8, 15, 16, 17, 31, 64, 96, 128, 130])
def test_dense_and_lut_dot_match_scalar(oracle, n):
    """simd.rs:278-322: the vector association agrees with the plain sum
    within the reference's own bar, 1e-4 + 1e-4*|want|."""
    a = _xorshift_stream(99 + n, 2 * n)
    x, y = a[:n], a[n:]
    want = np.float32(0)
    for i in range(n):
        want += x[i] * y[i]
    got = oracle.dense_dot(x, y)
    assert abs(got - want) <= 1e-4 + 1e-4 * abs(want)
    book = y.copy()
    idx = np.arange(n, dtype=np.uint32)
    assert oracle.lut_dot_u32(x, idx, book) == got


def test_fwht_is_self_inverse(oracle):
    """lib.rs:825-833."""
    buf = np.array([0.3, -1.2, 0.7, 2.1, -0.5, 0.9, 1.4, -2.0], np.float32)
    back = oracle.fwht(oracle.fwht(buf))
    np.testing.assert_allclose(back, buf, atol=1e-5)


def test_rotation_round_trips_and_preserves_norm(oracle):
    """lib.rs:835-849 (dim 768 = 512 + 256 blocks, seed 7, three rounds)."""
    from fixtures import next_f64_stream

    c = oracle.Codec(768, 2, 4, seed=7)
    v = (next_f64_stream(11, 768) * 2.0 - 1.0).astype(np.float32)
    back = c.rotate_inverse(c.rotate(v))
    np.testing.assert_allclose(back, v, atol=1e-4)
    assert abs(oracle.l2_norm(c.rotate(v)) - oracle.l2_norm(v)) < 1e-4


@pytest.mark.parametrize("bits", [4, 5, 6, 1, 2, 3])
def test_pack_unpack_round_trips(oracle, bits):
    """lib.rs:851-866."""
    rng = np.random.default_rng(123 + bits)
    idx = rng.integers(0, 1 << bits, 200).astype(np.uint16)
    packed = oracle.pack_indices(idx, bits)
    assert len(packed) == (200 * bits + 7) // 8
    np.testing.assert_array_equal(oracle.unpack_indices(packed, bits, 200), idx)


def test_unpack_survives_a_truncated_buffer(oracle):
    """lib.rs:868-887."""
    bits, n = 5, 64
    idx = (np.arange(n) & 31).astype(np.uint16)
    packed = oracle.pack_indices(idx, bits)
    for keep in [0, 1, 3, len(packed) // 2, len(packed) - 1]:
        out = oracle.unpack_indices(packed[:keep], bits, n)
        dec = keep * 8 // bits
        np.testing.assert_array_equal(out[:dec], idx[:dec])


def test_codes_only_matches_recon_ranking(oracle):
    """trellis.rs:2954-3004: scoring through windows (codes-only) and through a
    decoded x-bar (recon cache) rank the top-10 identically."""
    dim = 128
    db = oracle.rand_unit(200, dim, 17)
    qs = oracle.rand_unit(20, dim, 23)
    c = oracle.Codec(dim, 2, 12)
    idx = c.encode_batch(db)
    ids, _ = c.search_topk(idx, qs, 10)
    tab = c.table()
    for qi, q in enumerate(qs):
        q_r, _ = c.prepare_query(q)
        scores = []
        for i in range(200):
            w = c.windows(idx["codes"][i], int(idx["start"][i]))
            xbar = tab[w]
            scores.append(np.float32(oracle.dense_dot(q_r, xbar)) / idx["rescale"][i])
        order = sorted(range(200), key=lambda i: (-scores[i], i))[:10]
        assert list(ids[qi]) == order


def test_ivf_full_probe_recovers_flat_recall(oracle):
    """ivf.rs:855-909 (recon arm; codes-only scores identically): 400 x 128,
    16 lists, 8 bits per coordinate (M lowered from the default 12 to 8 to
    keep the CPU suite fast); nprobe = nlist loses nothing."""
    dim = 128
    db = oracle.rand_unit(400, dim, 31)
    qs = oracle.rand_unit(40, dim, 37)
    nlist = 16
    cen = oracle.kmeans(db, nlist, 42)
    asg = oracle.assign(db, cen)
    gold = oracle.exact_topk(db, qs, 10, cosine=True)
    c = oracle.Codec(dim, 8, 8)
    order = np.argsort(asg, kind="stable")
    off = np.zeros(nlist + 1, np.int64)
    np.add.at(off, asg.astype(np.int64) + 1, 1)
    off = np.cumsum(off)
    enc = c.ivf_encode(db[order], None, asg[order])
    ids_full, _ = c.ivf_search_topk(cen, off, order.astype(np.int64), enc, False, qs, nlist, 10)
    r_full = np.mean([len(set(gold[q]) & set(ids_full[q])) / 10 for q in range(40)])
    ids_1, _ = c.ivf_search_topk(cen, off, order.astype(np.int64), enc, False, qs, 1, 10)
    r_1 = np.mean([len(set(gold[q]) & set(ids_1[q])) / 10 for q in range(40)])
    assert r_full > 0.95 and r_1 <= r_full + 1e-9
    # flat scan over the same records ranks identically at full probe
    flat = c.encode_batch(db)
    ids_flat, _ = c.search_topk(flat, qs, 10)
    np.testing.assert_array_equal(ids_flat, ids_full)


def test_digest_is_order_independent(oracle):
    """trellis.rs:970-990: XOR-folded FNV-1a per record."""
    c = oracle.Codec(128, 2, 8)
    idx = c.encode_batch(oracle.rand_unit(50, 128, 5))
    d1 = oracle.digest(idx["codes"], idx["start"])
    perm = np.random.default_rng(0).permutation(50)
    d2 = oracle.digest(idx["codes"][perm], idx["start"][perm])
    assert d1 == d2 and d1 != 0


def test_candidate_scorer_agrees_with_search(oracle):
    """trellis.rs:2016-2086: prepare + score_at over every record gives the
    scores search ranks (the same estimator), 0.0 for a zero query, and the
    centered qm term per record."""
    dim = 64
    db = oracle.rand_unit(300, dim, 41)
    qs = oracle.rand_unit(6, dim, 43)
    qs[3] = 0.0
    for cen in (None, oracle.kmeans(db, 4, 42)):
        c = oracle.Codec(dim, 2, 8, centroids=cen)
        idx = c.encode_batch(db)
        pos = np.tile(np.arange(300, dtype=np.int64), len(qs))
        off = np.arange(len(qs) + 1, dtype=np.int64) * 300
        s = c.score_candidates(idx, qs, pos, off).reshape(len(qs), 300)
        ids, top = c.search_topk(idx, qs, 10)
        for q in range(len(qs)):
            if q == 3:
                assert np.all(s[q] == 0.0) and np.all(ids[q] == -1)
                continue
            order = sorted(range(300), key=lambda i: (-s[q, i], i))[:10]
            assert list(ids[q]) == order
            assert np.array_equal(s[q, ids[q]].view(np.uint32), top[q].view(np.uint32))
        # one query without offsets: the same numbers
        one = c.score_candidates(idx, qs[0], np.arange(300))
        assert np.array_equal(one.view(np.uint32), s[0].view(np.uint32))


def _unit(rows):
    n = np.linalg.norm(rows.astype(np.float64), axis=1, keepdims=True)
    return (rows / np.maximum(n, 1e-30)).astype(np.float32)


def test_sign_code_is_the_packed_sign_of_u_r(oracle):
    """trellis.rs:1084-1094: sign_code = pack_indices(u_r > 0, 1), dim/8 bytes."""
    dim = 128
    rows = oracle.rand_unit(40, dim, 7)
    c = oracle.Codec(dim, 2, 8)
    enc = c.encode_batch_signs(rows)
    plain = c.encode_batch(rows)
    assert np.array_equal(enc["codes"], plain["codes"])  # the field is inert for the codes
    for i in range(40):
        u_r = c.rotate(rows[i] / np.float32(oracle.l2_norm(rows[i])))
        bits = (u_r > 0).astype(np.uint16)
        assert np.array_equal(enc["signs"][i], oracle.pack_indices(bits, 1))


def test_shortlist_c_eq_n_matches_full_scan(oracle):
    """trellis.rs:3202-3249: at C = N nothing is pruned, so the two-stage
    search returns the plain codes-only top-10 (M lowered to 8)."""
    dim = 128
    db = oracle.rand_unit(200, dim, 31)
    c = oracle.Codec(dim, 2, 8)
    enc = c.encode_batch_signs(db)
    qs = oracle.rand_unit(20, dim, 37)
    a, sa = c.search_topk(enc, qs, 10)
    for asym in (False, True):
        b, sb = c.search_shortlist(enc, qs, 10, 200, asym=asym)
        assert np.array_equal(a, b) and np.array_equal(sa.view(np.uint32), sb.view(np.uint32))


def test_shortlist_recall_monotone_in_c(oracle):
    """trellis.rs:3251-3300: recall@10 against C = N never drops as C grows."""
    dim = 128
    db = oracle.rand_unit(500, dim, 41)
    c = oracle.Codec(dim, 2, 8)
    enc = c.encode_batch_signs(db)
    qs = oracle.rand_unit(30, dim, 43)
    gold, _ = c.search_shortlist(enc, qs, 10, 500)
    prev = 0.0
    for cs in (50, 100, 200, 500):
        got, _ = c.search_shortlist(enc, qs, 10, cs)
        r = np.mean([len(set(gold[q]) & set(got[q])) / 10 for q in range(30)])
        assert r >= prev - 1e-9
        prev = r
    assert prev == 1.0


def test_asymmetric_stage1_beats_binarizing_the_query(oracle):
    """trellis.rs:3136-3200: a tight cluster (0.8 e0 + 0.6 r, one centroid,
    C = 16): the asymmetric stage 1 keeps the exhaustive top-1 more often
    than the Hamming one (M lowered to 8)."""
    dim = 128
    base = np.zeros(dim, np.float32)
    base[0] = 1.0
    r = oracle.rand_unit(600, dim, 71)
    db = _unit(np.float32(0.8) * base + np.float32(0.6) * r)
    centroid = np.zeros(dim, np.float32)
    for v in db:
        centroid += v
    centroid = centroid / np.float32(600)
    c = oracle.Codec(dim, 2, 8, centroids=centroid[None, :])
    enc = c.encode_batch_signs(db)
    qs = oracle.rand_unit(150, dim, 73)
    exact, _ = c.search_shortlist(enc, qs, 1, 600, asym=True)
    ga, _ = c.search_shortlist(enc, qs, 1, 16, asym=True)
    gh, _ = c.search_shortlist(enc, qs, 1, 16, asym=False)
    assert (ga[:, 0] == exact[:, 0]).sum() > (gh[:, 0] == exact[:, 0]).sum()


@pytest.mark.parametrize("asym", [False, True])
def test_shortlist_stages_restated(oracle, asym):
    """trellis.rs:874-948 restated in numpy: stage-1 similarity (Hamming or
    the sequential masked sum, times rnorm under centering), the C best by
    (similarity desc, entry asc), then score() and top-k by (score desc,
    entry asc)."""
    dim, n, k, cs = 64, 150, 5, 12
    db = oracle.rand_unit(n, dim, 91)
    cen = oracle.kmeans(db, 3, 42)
    c = oracle.Codec(dim, 2, 6, centroids=cen)
    enc = c.encode_batch_signs(db)
    qs = oracle.rand_unit(4, dim, 93)
    ids, scores = c.search_shortlist(enc, qs, k, cs, asym=asym)
    bits = np.unpackbits(enc["signs"], axis=1)[:, :dim]
    for qi, q in enumerate(qs):
        q_r, _ = c.prepare_query(q)
        if asym:
            sims = []
            for i in range(n):
                s = np.float32(0.0)
                for t in range(dim):
                    s = np.float32(s + (q_r[t] if bits[i, t] else -q_r[t]))
                sims.append(s)
            sims = np.array(sims, np.float32)
        else:
            qb = (q_r > 0).astype(np.uint8)
            h = (bits != qb[None, :]).sum(axis=1)
            sims = np.float32(dim) - np.float32(2.0) * h.astype(np.float32)
        sims = enc["rnorm"] * sims
        keep = sorted(range(n), key=lambda i: (-sims[i], i))[:cs]
        sc = c.score_candidates(enc, q, np.array(keep, np.int64))
        order = sorted(range(cs), key=lambda j: (-sc[j], keep[j]))[:k]
        assert list(ids[qi]) == [keep[j] for j in order]
        assert np.array_equal(scores[qi].view(np.uint32), sc[order].view(np.uint32))


def test_ivf_shortlist_full_c_matches_ivf_search(oracle):
    """ivf.rs:52-60 + 229-239: with C at least the longest list, every probed
    list reranks all its entries, so the shortlist arm equals the codes arm;
    centered and uncentered lists."""
    dim, nlist = 64, 8
    db = oracle.rand_unit(800, dim, 95)
    qs = oracle.rand_unit(20, dim, 97)
    cen = oracle.kmeans(db, nlist, 42)
    asg = oracle.assign(db, cen)
    order = np.argsort(asg, kind="stable")
    off = np.zeros(nlist + 1, np.int64)
    np.add.at(off, asg.astype(np.int64) + 1, 1)
    off = np.cumsum(off)
    c = oracle.Codec(dim, 2, 8)
    for centered in (False, True):
        enc = c.ivf_encode_signs(db[order], cen if centered else None, asg[order])
        a, sa = c.ivf_search_topk(cen, off, order.astype(np.int64), enc, centered, qs, 3, 10)
        b, sb = c.ivf_search_shortlist(cen, off, order.astype(np.int64), enc, centered, qs, 3,
                                       10, 800)
        assert np.array_equal(a, b) and np.array_equal(sa.view(np.uint32), sb.view(np.uint32))
        s, _ = c.ivf_search_shortlist(cen, off, order.astype(np.int64), enc, centered, qs, 3,
                                      10, 20, asym=True)
        assert np.mean([len(set(a[q]) & set(s[q])) for q in range(20)]) > 5
