"""The coset-trellis oracle (oracle/uv_oracle_coset.c) against the
reference's own tests of src/coset_trellis.rs and src/e8.rs, and its Viterbi
against an exhaustive search over every path.

The reference ships no golden vectors for this arm, so its parity is
unpinned: these properties are what the restatement is checked against."""
from __future__ import annotations

import itertools

import numpy as np
import pytest

EPS = np.float32(1.1920929e-07)


def test_the_partition_is_eight_balanced_cosets(oracle):
    """coset_trellis.rs:534-563: a coset plus a sublattice point stays in the
    coset, and the eight cosets are balanced on the low-norm points."""
    raw = oracle.e8_enumerate(20.0)
    labels = np.array([oracle.coset_of(p) for p in raw])
    zero = raw[labels == 0]
    rng = np.random.default_rng(7)
    for _ in range(2000):
        a = raw[rng.integers(len(raw))]
        b = zero[rng.integers(len(zero))]
        assert oracle.coset_of(a + b) == oracle.coset_of(a)
    counts = np.bincount(labels, minlength=8)
    assert counts.min() / counts.max() > 0.85


def test_e8_points_and_nearest(oracle):
    """e8.rs: the enumeration holds the 240 roots of norm 2 (+ the origin) and
    every point has one parity and an even coordinate sum; e8_nearest returns
    a lattice point no farther than any enumerated one."""
    raw = oracle.e8_enumerate(2.0)
    assert len(raw) == 241
    for p in raw:
        assert len({int(v) & 1 for v in p}) == 1 and int(p.sum()) % 4 == 0
    pts = oracle.e8_enumerate(8.0).astype(np.float32) / 2
    rng = np.random.default_rng(3)
    for _ in range(200):
        y = (rng.standard_normal(8) * 0.8).astype(np.float32)
        x = oracle.e8_nearest(y)
        d = ((pts - y) ** 2).sum(1).min()
        assert ((x - y) ** 2).sum() <= d + 1e-5


@pytest.mark.parametrize("bits", [1, 2])
def test_nearest_in_coset_matches_the_exhaustive_scan(oracle, bits):
    """coset_trellis.rs:565-593."""
    q = oracle.Coset(8, bits)
    mean, std = q.scale()
    rng = np.random.default_rng(11 + bits)
    checked = 0
    for _ in range(500):
        y = (rng.standard_normal(8).astype(np.float32) * np.float32(std) + np.float32(mean))
        for c in range(8):
            fi, fd = q.nearest(c, y)
            si, sd = q.nearest(c, y, exhaustive=True)
            if fi != si:
                assert abs(fd - sd) < 1e-5
            checked += 1
    assert checked >= 4000


def test_books_are_the_lowest_norm_points_of_each_coset(oracle):
    """coset_trellis.rs:131-170: per coset, its 2^(8b-3) lowest points by
    (norm, lex), and the scaling statistics over their union."""
    q = oracle.Coset(16, 1)
    raw = oracle.e8_enumerate(6.0)
    keys = np.array([oracle.e8_key(p) for p in raw], np.uint64)
    labels = np.array([oracle.coset_of(p) for p in raw])
    books = q.books()
    for c in range(8):
        want = np.sort(keys[labels == c])[: q.per_coset]
        assert np.array_equal(books[c], want)
        pts = q.book_points(c)
        assert all(oracle.coset_of(p) == c for p in pts)
        assert q.index(c, pts[5]) == 5
    allp = np.concatenate([q.book_points(c) for c in range(8)]).astype(np.float64) / 2
    mean = allp.mean()
    std = np.sqrt(max((allp ** 2).mean() - mean * mean, 1e-12))
    assert q.scale() == pytest.approx((mean, std), rel=1e-6)


def test_a_record_decodes_to_the_path_the_encoder_chose(oracle):
    """coset_trellis.rs:595-615."""
    dim = 64
    q = oracle.Coset(dim, 2)
    v = np.array([((j * 37) % 101) / 101.0 - 0.5 for j in range(dim)], np.float32)
    out = q.reconstruct_unit(v)
    assert abs(np.linalg.norm(out) - 1.0) < 1e-4
    assert float(v @ out) / np.linalg.norm(v) > 0.5


def _path_costs(oracle, q, row):
    """Per block and coset: the nearest kept point's cost, as the encoder
    computes it (prep, rotation, standardization in f32)."""
    dim = q.dim
    rot = oracle.Codec(dim, 1, 1, rounds=3)
    n = max(np.float32(oracle.l2_norm(row)), EPS)
    u = (row / n).astype(np.float32)
    ur = rot.rotate(u)
    s = max(np.float32(oracle.std_about_mean(ur)), EPS)
    mean, std = q.scale()
    y = ((ur / np.float32(s)) * np.float32(std) + np.float32(mean)).astype(np.float32)
    return np.array([[q.nearest(c, y[b * 8:(b + 1) * 8])[1] for c in range(8)]
                     for b in range(dim // 8)], np.float32)


@pytest.mark.parametrize("mem,dim", [(1, 24), (2, 24), (3, 32), (4, 24)])
def test_viterbi_finds_a_cheapest_path(oracle, mem, dim):
    """coset_trellis.rs:343-381: the encoded path (start state, branches,
    cosets resolved by the state-parity rule) costs no more than any other
    path of the trellis, found by enumerating them all."""
    q = oracle.Coset(dim, 1, mem=mem)
    rng = np.random.default_rng(mem * 100 + dim)
    nb, mask = dim // 8, (1 << mem) - 1
    for _ in range(4):
        row = rng.standard_normal(dim).astype(np.float32)
        enc = q.encode_batch(row[None])
        cost = _path_costs(oracle, q, row)
        rec = enc["codes"][0]
        sb = (mem + 7) // 8
        start = int.from_bytes(bytes(rec[:sb]), "little")
        w = 2 + q.m_bits
        bitsr = "".join(f"{b:08b}" for b in rec[sb:])
        syms = [int(bitsr[i * w:(i + 1) * w], 2) for i in range(nb)]

        def walk(st, brs):
            tot = np.float32(0.0)
            for b, br in enumerate(brs):
                c = ((bin(st).count("1") & 1) << 2) | br
                tot = np.float32(tot + cost[b, c])
                st = ((st << 2) | br) & mask
            return tot

        got = walk(start, [s >> q.m_bits for s in syms])
        best = min(walk(s0, brs) for s0 in range(1 << mem)
                   for brs in itertools.product(range(4), repeat=nb))
        assert got == best


def test_search_finds_each_record_first(oracle):
    """coset_trellis.rs:471-497: a record's own vector scores it about 1 and
    ranks it first; ties keep insertion order; unfilled slots are empty."""
    q = oracle.Coset(32, 2)
    rng = np.random.default_rng(5)
    base = rng.standard_normal((300, 32)).astype(np.float32)
    enc = q.encode_batch(base)
    ids, sc = q.search(enc, base[:20], 10)
    assert np.array_equal(ids[:, 0], np.arange(20))
    assert np.all(np.abs(sc[:, 0] - 1.0) < 0.05)
    assert np.all(np.diff(sc, axis=1) <= 0)
    dup = {k: np.concatenate([v, v]) for k, v in enc.items()}
    ids2, sc2 = q.search(dup, base[:3], 4)
    assert np.array_equal(ids2[:, 0], np.arange(3)) and np.array_equal(ids2[:, 1], np.arange(300, 303))
    ids3, sc3 = q.search({k: v[:2] for k, v in enc.items()}, base[:1], 4)
    assert list(ids3[0, 2:]) == [-1, -1] and np.all(np.isneginf(sc3[0, 2:]))


def test_mem_bytes_and_record_length(oracle):
    """coset_trellis.rs:498-504: code bytes (start state + packed symbols) +
    4 + the centering bytes, per record."""
    q = oracle.Coset(128, 2, mem=12)
    assert q.code_len == 2 + (16 * 15 + 7) // 8
    assert q.mem_bytes(10) == 10 * (q.code_len + 4)
    qc = oracle.Coset(128, 2, mem=12, centroids=np.zeros((300, 128), np.float32))
    assert qc.mem_bytes(10) == 10 * (q.code_len + 4 + 4 + 2)


def test_rejects_unsupported_shapes(oracle):
    """coset_trellis.rs:121-130: dim % 8 == 0 and bits in 1..=3."""
    for dim, bits in [(12, 2), (16, 0), (16, 4)]:
        with pytest.raises(ValueError):
            oracle.Coset(dim, bits)
