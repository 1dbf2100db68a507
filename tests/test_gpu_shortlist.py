"""The 1-bit companion shortlist (csrc/shortlist.cu) against the oracle
(trellis.rs:841-948, ivf.rs:52-60): sign codes byte-identical, flat and IVF
searches bit-identical for both stage-1 scorers, with and without the rnorm
weight, centered and uncentered; C >= N equals the plain scan; index files
keep the shortlist."""
from __future__ import annotations

import numpy as np
import pytest

from fixtures import rand_rows

pytestmark = pytest.mark.gpu


def same(a, b):
    ia, sa = a
    ib, sb = b
    assert np.array_equal(np.asarray(ia), np.asarray(ib))
    assert np.array_equal(np.asarray(sa, np.float32).view(np.uint32),
                          np.asarray(sb, np.float32).view(np.uint32))


def flat_pair(uv, oracle, rows, dim, bits, mem, c, asym, rnorm, cen=None):
    codec = uv.Codec(dim, bits, mem)
    index = uv.Index(codec)
    if cen is not None:
        index.set_centroids(cen)
    index.set_shortlist(c, asym=asym, rnorm=rnorm)
    index.add_batch(rows)
    oc = oracle.Codec(dim, bits, mem, centroids=cen)
    enc = oc.encode_batch_signs(rows)
    e = index.export()
    assert np.array_equal(e["codes"], enc["codes"]) and np.array_equal(e["start"], enc["start"])
    assert np.array_equal(index.export_signs(), enc["signs"])
    return index, oc, enc


@pytest.mark.parametrize("asym", [False, True])
@pytest.mark.parametrize("centered", [False, True])
def test_flat_shortlist_bit_exact(uv, oracle, asym, centered):
    dim, n = 128, 6000
    rows = rand_rows(n, dim, 71) * np.float32(2.0)
    queries = rand_rows(40, dim, 72)
    queries[5] = 0.0  # degenerate: no results
    cen = oracle.kmeans(rows, 8, 42) if centered else None
    for rnorm in (True, False):
        for c in (16, 100, 512):
            index, oc, enc = flat_pair(uv, oracle, rows, dim, 2, 8, c, asym, rnorm, cen)
            for k in (1, 10, 64):
                got = index.search(queries, k)
                ref = oc.search_shortlist(enc, queries, k, c, asym=asym, weight=rnorm)
                same(got, ref)
                assert np.all(got[0][5] == -1)


@pytest.mark.parametrize("dim,bits,mem", [(64, 1, 10), (128, 4, 5), (96, 3, 6), (256, 2, 8)])
def test_flat_shortlist_widths(uv, oracle, dim, bits, mem):
    rows = rand_rows(3000, dim, 73)
    queries = rand_rows(16, dim, 74)
    for asym in (False, True):
        index, oc, enc = flat_pair(uv, oracle, rows, dim, bits, mem, 200, asym, True)
        same(index.search(queries, 10), oc.search_shortlist(enc, queries, 10, 200, asym=asym))


def test_c_at_least_n_is_the_plain_scan(uv, oracle):
    """trellis.rs:3202-3249: C = N prunes nothing."""
    rows = rand_rows(500, 128, 75)
    queries = rand_rows(20, 128, 76)
    codec = uv.Codec(128, 2, 8)
    plain = uv.Index(codec)
    plain.add_batch(rows)
    comp = uv.Index(codec)
    comp.set_shortlist(1)
    comp.add_batch(rows)
    assert comp.export_signs().shape == (500, 16)
    with pytest.raises(uv.UVError):
        plain.export_signs()
    comp.set_shortlist(500)
    same(plain.search(queries, 10), comp.search(queries, 10))
    comp.set_shortlist(499)  # one short of N: the shortlist kernel
    oc = oracle.Codec(128, 2, 8)
    enc = oc.encode_batch_signs(rows)
    same(comp.search(queries, 10), oc.search_shortlist(enc, queries, 10, 499))
    # the sign code is counted in mem_bytes (trellis.rs:2196)
    assert comp.mem_bytes() == plain.mem_bytes() + 500 * 16


def test_large_flat_shortlist(uv, oracle):
    rows = rand_rows(60_000, 128, 77)
    queries = rand_rows(24, 128, 78)
    for c in (1024, 4096):
        index, oc, enc = flat_pair(uv, oracle, rows, 128, 2, 8, c, False, True)
        same(index.search(queries, 100), oc.search_shortlist(enc, queries, 100, c))
    index.clear()
    with pytest.raises(uv.UVError) as e:
        index.set_shortlist(5000)
        index.add_batch(rows)
        index.search(queries, 10)
    assert e.value.code == 5


def test_shortlist_switch_needs_an_empty_index(uv):
    codec = uv.Codec(64, 2, 6)
    index = uv.Index(codec)
    index.add_batch(rand_rows(100, 64, 79))
    with pytest.raises(uv.UVError) as e:
        index.set_shortlist(10)
    assert e.value.code == 1
    index.clear()
    index.set_shortlist(10)
    index.add_batch(rand_rows(100, 64, 79))
    index.set_shortlist(20, asym=True)  # c and the scorer may change while on


def ivf_pair(uv, oracle, rows, nlist, centered, c, asym, rnorm, dim=64):
    cen = oracle.kmeans(rows, nlist, 42)
    codec = uv.Codec(dim, 2, 8)
    ivf = uv.IvfIndex(codec, cen, centered=centered)
    ivf.set_shortlist(c, asym=asym, rnorm=rnorm)
    ivf.build(rows)
    e = ivf.export()
    oc = oracle.Codec(dim, 2, 8)
    asg = oracle.assign(rows, cen)
    order = np.argsort(asg, kind="stable")
    enc = oc.ivf_encode_signs(rows[order], cen if centered else None, asg[order])
    assert np.array_equal(e["codes"], enc["codes"])
    assert np.array_equal(ivf.export_signs(), enc["signs"])
    return ivf, oc, enc, cen, e


@pytest.mark.parametrize("asym", [False, True])
@pytest.mark.parametrize("centered", [False, True])
def test_ivf_shortlist_bit_exact(uv, oracle, asym, centered):
    rows = rand_rows(8000, 64, 80)
    queries = rand_rows(48, 64, 81)
    queries[3] = 0.0
    for rnorm in (True, False):
        ivf, oc, enc, cen, e = ivf_pair(uv, oracle, rows, 32, centered, 24, asym, rnorm)
        for nprobe in (1, 4, 32):
            got = ivf.search(queries, 10, nprobe)
            ref = oc.ivf_search_shortlist(cen, e["list_off"], e["ids"], enc, centered, queries,
                                          nprobe, 10, 24, asym=asym, weight=rnorm)
            same(got, ref)


def test_ivf_shortlist_with_empty_lists_and_full_c(uv, oracle):
    """Lists with no entries contribute nothing; C above every list length
    reranks whole lists, which equals the codes arm (ivf.rs:52-60)."""
    rows = rand_rows(600, 64, 82)
    queries = rand_rows(16, 64, 83)
    cen = np.concatenate([oracle.kmeans(rows, 6, 42), rand_rows(2, 64, 84) * 50], axis=0)
    codec = uv.Codec(64, 2, 8)
    plain = uv.IvfIndex(codec, cen, centered=True)
    plain.build(rows)
    sl = uv.IvfIndex(codec, cen, centered=True)
    sl.set_shortlist(600)
    sl.build(rows)
    for nprobe in (2, 8):
        same(plain.search(queries, 10, nprobe), sl.search(queries, 10, nprobe))


def test_shortlist_survives_index_files(uv, oracle, tmp_path):
    rows = rand_rows(3000, 64, 85)
    queries = rand_rows(20, 64, 86)
    codec = uv.Codec(64, 2, 8)
    index = uv.Index(codec)
    index.set_shortlist(50, asym=True)
    index.add_batch(rows)
    index.save(tmp_path / "f.uvb")
    back = uv.Index.load(codec, tmp_path / "f.uvb")
    assert np.array_equal(back.export_signs(), index.export_signs())
    same(back.search(queries, 10), index.search(queries, 10))
    ivf, oc, enc, cen, e = ivf_pair(uv, oracle, rows, 16, True, 12, False, True)
    ivf.save(tmp_path / "i.uvb")
    back = uv.IvfIndex.load(codec, tmp_path / "i.uvb")
    assert np.array_equal(back.export_signs(), ivf.export_signs())
    same(back.search(queries, 10, 4), ivf.search(queries, 10, 4))
