"""Index files (csrc/capi_store.cu): a saved and reloaded index holds the same
records and answers every search identically; damaged files, files of another
codec configuration or of another index kind are refused with UV_EINVAL."""
from __future__ import annotations

import numpy as np
import pytest

from fixtures import rand_rows

pytestmark = pytest.mark.gpu


def same_export(a, b):
    assert a.keys() == b.keys()
    for key in a:
        x, y = np.asarray(a[key]), np.asarray(b[key])
        assert np.array_equal(x.view(np.uint8), y.view(np.uint8)), key


def test_flat_round_trip(uv, oracle, tmp_path):
    rows = rand_rows(5000, 128, 41) * np.float32(3.0)
    queries = rand_rows(64, 128, 42)
    codec = uv.Codec(128, 2, 8)
    index = uv.Index(codec)
    index.add(np.arange(5000, dtype=np.int64) * 7 + 3, rows)
    path = tmp_path / "flat.uvb"
    index.save(path)
    back = uv.Index.load(codec, path)
    assert len(back) == 5000
    same_export(index.export(), back.export())
    assert back.digest() == index.digest()
    for mips in (False, True):
        a, b = index.search(queries, 25, mips=mips), back.search(queries, 25, mips=mips)
        assert np.array_equal(a[0], b[0]) and np.array_equal(a[1].view(np.uint32),
                                                             b[1].view(np.uint32))
    # a reloaded index keeps growing like the original
    more = rand_rows(300, 128, 43)
    index.add_batch(more)
    back.add_batch(more)
    assert back.digest() == index.digest()


def test_flat_centered_and_empty(uv, oracle, tmp_path):
    rows = rand_rows(2000, 64, 44)
    codec = uv.Codec(64, 2, 6)
    index = uv.Index(codec)
    index.set_centroids(oracle.kmeans(rows, 8, 42))
    index.add_batch(rows)
    index.save(tmp_path / "c.uvb")
    back = uv.Index.load(codec, tmp_path / "c.uvb")
    same_export(index.export(), back.export())
    q = rand_rows(16, 64, 45)
    a, b = index.search(q, 10), back.search(q, 10)
    assert np.array_equal(a[0], b[0]) and np.array_equal(a[1].view(np.uint32), b[1].view(np.uint32))
    empty = uv.Index(codec)
    empty.save(tmp_path / "e.uvb")
    assert len(uv.Index.load(codec, tmp_path / "e.uvb")) == 0


def test_ivf_round_trip(uv, oracle, tmp_path):
    rows = rand_rows(4000, 64, 46)
    cen = oracle.kmeans(rows, 16, 42)
    codec = uv.Codec(64, 2, 6)
    ivf = uv.IvfIndex(codec, cen, centered=True)
    ivf.build(rows)
    ivf.save(tmp_path / "ivf.uvb")
    back = uv.IvfIndex.load(codec, tmp_path / "ivf.uvb")
    assert len(back) == 4000 and back.nlist == 16
    same_export(ivf.export(), back.export())
    q = rand_rows(32, 64, 47)
    for nprobe in (1, 5, 16):
        a, b = ivf.search(q, 10, nprobe), back.search(q, 10, nprobe)
        assert np.array_equal(a[0], b[0]) and np.array_equal(a[1].view(np.uint32),
                                                             b[1].view(np.uint32))


def test_damaged_and_foreign_files_are_refused(uv, oracle, tmp_path):
    rows = rand_rows(500, 64, 48)
    codec = uv.Codec(64, 2, 6)
    index = uv.Index(codec)
    index.add_batch(rows)
    good = tmp_path / "good.uvb"
    index.save(good)
    data = good.read_bytes()

    def refused(payload, codec_=codec, kind=uv.Index):
        bad = tmp_path / "bad.uvb"
        bad.write_bytes(payload)
        with pytest.raises(uv.UVError) as e:
            kind.load(codec_, bad)
        assert e.value.code == 1

    flipped = bytearray(data)
    flipped[len(data) // 2] ^= 0x10
    refused(bytes(flipped))                     # checksum
    refused(data[: len(data) - 9])              # truncated
    refused(data + b"\0")                       # trailing bytes
    refused(b"NOTANIDX" + data[8:])             # magic
    refused(data, codec_=uv.Codec(64, 2, 7))    # another configuration
    refused(data, codec_=uv.Codec(64, 2, 6, seed=7))
    refused(data, kind=uv.IvfIndex)             # another kind of index
    with pytest.raises(uv.UVError):
        uv.Index.load(codec, tmp_path / "missing.uvb")
