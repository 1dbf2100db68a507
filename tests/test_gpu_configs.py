"""Parity at the shapes of the measured configurations, on the GPU against the
oracle, at sizes the oracle finishes in seconds:

- the encoder memory sweep: d = 128, b = 2, N(0,1) rows, every state-bit
  count of the sweep (2, 4, 8, 12, 16; M = 16 is one thread-block cluster of
  16 CTAs per row);
- the IVF configuration: rows of 1536 coordinates zero-padded to 2048, unit
  vectors from a Gaussian mixture, nlist >= 256 (tensor-core k-means
  assignment and probe), centered lists, a posting list longer than one scan
  range (range splitting), empty lists, nprobe 1 / 16 / 64, top-10;
- the wide-row configuration: 960 coordinates padded to 1024 with a
  per-coordinate mean drift, b = 1, 2, 4, MIPS top-10 through the K-chunked
  tensor-core prefilter.
The 1M x 10k flat configuration is checked inside the benchmark itself
(its `parity` entry: the oracle's top-100 for a sample of the timed queries
over all 1M GPU records, and the first 8,192 records byte for byte)."""
from __future__ import annotations

import numpy as np
import pytest

from test_gpu_ivf import bits_equal, clustered, oracle_lists

pytestmark = pytest.mark.gpu


def _bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


@pytest.mark.parametrize("mem,n", [(2, 2000), (4, 2000), (8, 1000), (12, 200), (16, 32)])
def test_encode_sweep_cells_bit_exact(uv, oracle, mem, n):
    rng = np.random.default_rng(1)
    rows = rng.standard_normal((n, 128), dtype=np.float32)
    g = uv.Codec(128, 2, mem)
    o = oracle.Codec(128, 2, mem)
    got = g.encode(rows)
    want = o.encode_batch(rows)
    np.testing.assert_array_equal(got["codes"], want["codes"])
    np.testing.assert_array_equal(got["start"], want["start"])
    np.testing.assert_array_equal(_bits(got["rescale"]), _bits(want["rescale"]))


def _ivf_corpus(n_cluster, n_dup, nq, d, d_pad, seed):
    """Gaussian-mixture units (64 centres, std 0.3, renormalized) in the
    first d of d_pad coordinates, plus n_dup copies of one row (they all land
    in one posting list: k-means keeps duplicated centroids, the first one
    wins every assignment) and queries near both."""
    rng = np.random.default_rng(seed)
    c = rng.standard_normal((64, d)).astype(np.float32)
    c /= np.linalg.norm(c, axis=1, keepdims=True)
    x = np.zeros((n_cluster + n_dup + nq, d_pad), np.float32)
    v = c[rng.integers(0, 64, n_cluster + nq)] + np.float32(0.3) * rng.standard_normal(
        (n_cluster + nq, d), dtype=np.float32)
    v /= np.linalg.norm(v, axis=1, keepdims=True)
    x[:n_cluster, :d] = v[:n_cluster]
    x[n_cluster:n_cluster + n_dup, :d] = v[0]
    x[n_cluster + n_dup:, :d] = v[n_cluster:]
    x[n_cluster + n_dup:n_cluster + n_dup + nq // 4, :d] += np.float32(0.05) * v[0]
    base, queries = x[:n_cluster + n_dup], x[n_cluster + n_dup:]
    perm = rng.permutation(len(base))
    return base[perm], queries


def test_ivf_configuration_shape(uv, oracle):
    d, d_pad, nlist = 1536, 2048, 256
    base, queries = _ivf_corpus(17_000, 3_000, 96, d, d_pad, 4)
    cen = oracle.kmeans(base, nlist, seed=42, iters=2)
    got_cen = uv.kmeans(base, nlist, seed=42, iters=2)
    assert bits_equal(got_cen, cen)
    assign = oracle.assign(base, cen)
    assert np.array_equal(uv.ivf_assign(base, cen), assign)
    sizes = np.bincount(assign, minlength=nlist)
    assert sizes.max() > 2048 and (sizes == 0).any()  # range splitting, empty lists
    ocodec = oracle.Codec(d_pad, 2, 8)
    off, ids, lists = oracle_lists(oracle, ocodec, base, cen, assign, True)
    ivf = uv.IvfIndex(uv.Codec(d_pad, 2, 8), cen, centered=True)
    ivf.build(base)
    ex = ivf.export()
    assert np.array_equal(ex["list_off"], off) and np.array_equal(ex["ids"], ids)
    assert np.array_equal(ex["codes"], lists["codes"])
    assert np.array_equal(ex["start"], lists["start"])
    assert bits_equal(ex["rescale"], lists["rescale"]) and bits_equal(ex["rnorm"], lists["rnorm"])
    for nprobe in (1, 16, 64):
        got = ivf.probe(queries, nprobe)
        want = np.stack([oracle.ivf_probe(cen, q, nprobe) for q in queries])
        assert np.array_equal(got, want), nprobe
        gi, gs = ivf.search(queries, 10, nprobe)
        wi, ws = ocodec.ivf_search_topk(cen, off, ids, lists, True, queries, nprobe, 10)
        assert np.array_equal(gi, wi), nprobe
        assert bits_equal(gs, ws), nprobe


@pytest.mark.parametrize("bits", [1, 2, 4])
def test_wide_row_configuration_shape(uv, oracle, bits):
    n, nq, d, d_pad = 8192, 24, 960, 1024
    rng = np.random.default_rng(bits)
    x = np.zeros((n + nq, d_pad), np.float32)
    x[:, :d] = rng.random((n + nq, d), dtype=np.float32) + \
        np.float32(0.5) * (np.arange(d, dtype=np.float32) / np.float32(959))
    base, qs = x[:n], x[n:]
    g = uv.Codec(d_pad, bits, 8)
    ix = uv.Index(g)
    ix.add_batch(base)
    o = oracle.Codec(d_pad, bits, 8)
    enc = o.encode_batch(base)
    ex = ix.export()
    np.testing.assert_array_equal(ex["codes"], enc["codes"])
    np.testing.assert_array_equal(ex["start"], enc["start"])
    norms = oracle.l2_norms(base)
    try:
        uv.set_tuning("tc_scan", 2)  # the prefilter wherever it is built
        ids, scores = ix.search(qs, 10, mips=True)
    finally:
        uv.set_tuning("tc_scan", 0)
    wids, wscores = o.search_topk(enc, qs, 10, norms=norms)
    np.testing.assert_array_equal(ids, wids)
    np.testing.assert_array_equal(_bits(scores), _bits(wscores))
