"""CPU-only checks of the product side: the library loads and exports every
entry point the header declares; the host sharding and top-k merge logic
(including a world_size-2 gloo run); the bench's input generator."""
from __future__ import annotations

import os
import re
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parents[1]


def header_symbols():
    text = (REPO / "include" / "ultravec_b200.h").read_text()
    return sorted(set(re.findall(r"^\s*(?:int|void|const char \*)\s*(uv_\w+)\s*\(", text, re.M)))


def test_library_exports_every_declared_symbol(uv):
    declared = header_symbols()
    assert len(declared) >= 30
    lib = uv.lib()
    missing = [s for s in declared if not hasattr(lib, s)]
    assert not missing, missing
    assert sorted(declared) == sorted(uv.SYMBOLS)
    assert lib.uv_abi_version() == 1


def test_codec_create_without_gpu_fails_cleanly(uv):
    """No panic across the ABI: without a device the call returns a status."""
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    with pytest.raises(uv.UVError) as e:
        uv.Codec(128, 2, 8)
    assert e.value.code in (1, 3)


def test_bad_configs_are_rejected_before_any_device_work(uv):
    import ctypes as C

    cfg = uv.binding.uv_config()
    for dim, bits, mem in [(0, 2, 8), (128, 0, 8), (128, 5, 8), (128, 2, 0), (128, 4, 21)]:
        uv.lib().uv_config_default(C.byref(cfg), dim, bits, mem)
        h = C.c_void_p()
        assert uv.lib().uv_codec_create(C.byref(cfg), C.byref(h)) == 1
        assert uv.lib().uv_last_error()


def test_null_handles_are_refused_without_device_work(uv):
    """Every entry point whose first argument is a handle returns UV_EINVAL
    with a message for a null handle (other pointers null, sizes 0), before
    any device work; the destroy calls accept null like free(NULL).  Nothing
    crashes or aborts across the ABI."""
    import ctypes as C

    lib = uv.lib()
    ints = (C.c_int32, C.c_int64, C.c_uint64, C.c_float, C.c_int)
    checked = 0
    for name in uv.SYMBOLS:
        fn = getattr(lib, name)
        ats = fn.argtypes or []
        if not ats or ats[0] is not C.c_void_p:
            continue
        args = [0 if t in ints else None for t in ats]
        rc = fn(*args)
        if name.endswith("_destroy"):
            assert rc == 0, name
        else:
            assert rc == 1, (name, rc)
            assert lib.uv_last_error(), name
        checked += 1
    assert checked >= 60


def test_merges_of_no_rows_need_no_buffers_or_device(uv):
    """A rank whose query slice is empty (fewer queries than ranks) merges
    zero rows: the merges return UV_OK for null buffers and touch no device,
    while bad sizes and null buffers with rows are still refused."""
    lib = uv.lib()
    assert lib.uv_topk_merge_packed(0, None, 0, 4, 10, 10, 0, 10, None, None, None) == 0
    assert lib.uv_topk_merge(0, None, None, 0, 4, 10, 10, None, None, None) == 0
    assert lib.uv_topk_merge_packed(0, None, 3, 4, 10, 10, 30, 10, None, None, None) == 1
    assert lib.uv_topk_merge(0, None, None, 0, 4, 10, 41, None, None, None) == 1
    assert lib.uv_topk_pack(0, None, None, 0, None, None) == 0
    assert lib.uv_topk_unpack(0, None, 0, None, None, None) == 0


def test_shard_ranges_partition_the_rows(uv):
    from ultravec_ann_b200.shard import shard_range

    for n in (0, 1, 7, 1000, 1_000_000):
        for world in (1, 2, 3, 8):
            spans = [shard_range(n, r, world) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            sizes = [hi - lo for lo, hi in spans]
            assert max(sizes) - min(sizes) <= 1


def test_host_merge_orders_by_score_then_id(uv):
    from ultravec_ann_b200.shard import merge_host

    ids = np.array([[[5, 9, -1], [2, 3, 4]]], np.int64)
    sc = np.array([[[3.0, 1.0, -np.inf], [3.0, 2.0, 1.0]]], np.float32)
    oi, os_ = merge_host(ids, sc, 4)
    assert list(oi[0]) == [2, 5, 3, 4]
    assert list(os_[0]) == [3.0, 3.0, 2.0, 1.0]


def _gloo_worker(rank, world, port, result_dir):
    import torch
    import torch.distributed as dist

    import sys

    sys.path.insert(0, str(REPO / "oracle"))
    sys.path.insert(0, str(REPO / "tests"))
    sys.path.insert(0, str(REPO))
    import oracle as O
    from fixtures import rand_rows
    from ultravec_ann_b200_loader import load

    uv = load()
    from ultravec_ann_b200.shard import gather_topk, merge_host, shard_range

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    rows = rand_rows(600, 64, 3)
    qs = rand_rows(12, 64, 4)
    lo, hi = shard_range(len(rows), rank, world)
    codec = O.Codec(64, 2, 6)
    enc = codec.encode_batch(rows[lo:hi])
    ids, sc = codec.search_topk(enc, qs, 10, norms=O.l2_norms(rows[lo:hi]))
    ids = np.where(ids >= 0, ids + lo, -1)
    g_ids, g_sc = gather_topk(torch.from_numpy(ids), torch.from_numpy(sc), 10, dist, merge_host)
    if rank == 0:
        full = codec.encode_batch(rows)
        want_ids, want_sc = codec.search_topk(full, qs, 10, norms=O.l2_norms(rows))
        ok = np.array_equal(g_ids.numpy(), want_ids) and np.array_equal(
            g_sc.numpy().view(np.uint32), want_sc.view(np.uint32))
        Path(result_dir, "ok").write_text("1" if ok else "0")
    dist.barrier()
    dist.destroy_process_group()


def test_sharded_search_equals_unsharded_with_two_gloo_ranks(tmp_path):
    """world_size 2 on CPU: shard, local top-k (the oracle stands in for the
    device scan), all-gather, merge == the top-k of the whole index."""
    import socket

    import torch.multiprocessing as mp

    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    mp.start_processes(_gloo_worker, args=(2, port, str(tmp_path)), nprocs=2, join=True,
                       start_method="spawn")
    assert (tmp_path / "ok").read_text() == "1"


def _gloo_protocol_worker(rank, world, port, result_dir):
    """One rank of the sharded flat search protocol (shard.sharded_search)
    on gloo: the oracle stands in for the device phases (bounds = the
    shard's exact top-k scores, a valid lower bound for k distinct records;
    finish = its top-k cut at the shared threshold) and host routines for
    pack / merge."""
    import torch
    import torch.distributed as dist

    import sys

    sys.path.insert(0, str(REPO / "oracle"))
    sys.path.insert(0, str(REPO))
    import oracle as O
    from ultravec_ann_b200_loader import load

    load()
    from ultravec_ann_b200.shard import (merge_packed_host, pack_host, shard_range,
                                         sharded_search, unpack_host)

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    rows = O.rand_unit(700, 64, 61) * np.float32(3.0)
    rows[5] = rows[600]  # an exact tie across shards, broken by id
    qs = O.rand_unit(16, 64, 62)
    k = 10
    codec = O.Codec(64, 2, 8)
    lo, hi = shard_range(len(rows), rank, world)
    enc = codec.encode_batch(rows[lo:hi])
    norms = O.l2_norms(rows[lo:hi])

    class StandIn:
        def __init__(self):
            ids, sc = codec.search_topk(enc, qs, k, norms=norms)
            self.ids = np.where(ids >= 0, ids + lo, -1)
            self.sc = sc
            self.bounds = torch.from_numpy(sc.copy())
            self.theta = None

        def set_bounds(self, gathered, n):
            g = gathered.numpy().reshape(n, len(qs), k).transpose(1, 0, 2).reshape(len(qs), -1)
            self.theta = -np.sort(-g, axis=1)[:, k - 1]

        def finish(self, deferred=False):
            keep = self.sc >= self.theta[:, None]
            self.want = (np.where(keep, self.ids, -1),
                         np.where(keep, self.sc, -np.inf).astype(np.float32))
            self.out = (torch.from_numpy(self.want[0].copy()),
                        torch.from_numpy(self.want[1].copy()))
            if rank == 0:
                # rank 0's first query "overflowed": its deferred lists are
                # wrong until check() rewrites them, as the library does
                self.out[0][0] = -1
                self.out[1][0] = -np.inf
            return self.out

        def check(self):
            self.out[0][:] = torch.from_numpy(self.want[0])
            self.out[1][:] = torch.from_numpy(self.want[1])
            return rank == 0

        def close(self):
            pass

    g_ids, g_sc = sharded_search(lambda n: StandIn(), k, dist, pack_host, unpack_host,
                                 merge_packed_host, deferred=True)
    full = codec.encode_batch(rows)
    want_ids, want_sc = codec.search_topk(full, qs, k, norms=O.l2_norms(rows))
    ok = np.array_equal(g_ids.numpy(), want_ids) and np.array_equal(
        g_sc.numpy().view(np.uint32), want_sc.view(np.uint32))
    Path(result_dir, f"ok{rank}").write_text("1" if ok else "0")
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3, 4])
def test_sharded_search_protocol_with_gloo_ranks(tmp_path, world):
    """The flat multi-GPU protocol on CPU ranks: bounds all-gathered, shared
    threshold, lists packed, all-to-all of query slices (uneven at world 3),
    per-slice merge, all-gather -- every rank ends with the unsharded top-k;
    one rank's deferred lists are rewritten by its outcome check (an
    overflowed query), and every rank merges again."""
    import socket

    import torch.multiprocessing as mp

    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    mp.start_processes(_gloo_protocol_worker, args=(world, port, str(tmp_path)), nprocs=world,
                       join=True, start_method="spawn")
    for r in range(world):
        assert (tmp_path / f"ok{r}").read_text() == "1"


def test_ivf_list_owners_balance_bytes(uv):
    from ultravec_ann_b200.shard import ivf_list_owners, ivf_owned_rows

    rng = np.random.default_rng(5)
    sizes = rng.geometric(1 / 300, 4096)
    for world in (1, 2, 4, 8):
        own = ivf_list_owners(sizes, world)
        load = np.bincount(own, weights=sizes, minlength=world)
        assert set(own.tolist()) == set(range(world))
        assert load.max() - load.min() <= sizes.max()
        assert np.array_equal(own, ivf_list_owners(sizes, world))
    assign = rng.integers(0, 16, 500)
    own = ivf_list_owners(np.bincount(assign, minlength=16), 3)
    parts = [ivf_owned_rows(assign, own, r) for r in range(3)]
    assert np.array_equal(np.sort(np.concatenate(parts)), np.arange(500))


def _gloo_ivf_worker(rank, world, port, result_dir):
    import torch
    import torch.distributed as dist

    import sys

    sys.path.insert(0, str(REPO / "oracle"))
    sys.path.insert(0, str(REPO))
    import oracle as O
    from ultravec_ann_b200_loader import load

    load()
    from ultravec_ann_b200.shard import (gather_topk, ivf_list_owners, ivf_owned_rows,
                                         ivf_sharded_search, merge_host, merge_packed_host,
                                         pack_host, unpack_host)

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    dim, nlist = 64, 12
    db = O.rand_unit(900, dim, 41)
    qs = O.rand_unit(15, dim, 43)
    cen = O.kmeans(db, nlist, 42)
    asg = O.assign(db, cen)
    c = O.Codec(dim, 2, 8)

    def ivf_search(rows_idx, centered):
        sub = asg[rows_idx]
        order = rows_idx[np.argsort(sub, kind="stable")]
        off = np.zeros(nlist + 1, np.int64)
        np.add.at(off, asg[order].astype(np.int64) + 1, 1)
        off = np.cumsum(off)
        enc = c.ivf_encode(db[order], cen if centered else None, asg[order])
        return c.ivf_search_topk(cen, off, order.astype(np.int64), enc, centered, qs, 4, 10)

    owners = ivf_list_owners(np.bincount(asg, minlength=nlist), world)
    ok = True
    for centered in (False, True):
        ids, sc = ivf_search(ivf_owned_rows(asg, owners, rank), centered)
        g_ids, g_sc = gather_topk(torch.from_numpy(ids), torch.from_numpy(sc), 10, dist,
                                  merge_host)
        want_ids, want_sc = ivf_search(np.arange(len(db)), centered)
        if rank == 0:
            ok &= np.array_equal(g_ids.numpy(), want_ids) and np.array_equal(
                g_sc.numpy().view(np.uint32), want_sc.view(np.uint32))

        # the probe split by query slices, the lists shared, each rank
        # scanning its own lists (the oracle stands in for the device index)
        class Shard:
            def __init__(self, rows_idx):
                self.rows_idx = rows_idx

            def probe(self, q, nprobe):
                return torch.from_numpy(np.stack(
                    [np.asarray(O.ivf_probe(cen, x, nprobe), np.int32) for x in q])
                    if len(q) else np.zeros((0, nprobe), np.int32))

            def search_lists(self, q, k, lists):
                full = np.stack([np.asarray(O.ivf_probe(cen, x, 4), np.int32) for x in q])
                assert np.array_equal(np.asarray(lists), full)
                i, s = ivf_search(self.rows_idx, centered)
                return torch.from_numpy(i), torch.from_numpy(s)

        s_ids, s_sc = ivf_sharded_search(Shard(ivf_owned_rows(asg, owners, rank)), qs, 10, 4,
                                         dist, pack_host, unpack_host, merge_packed_host)
        ok &= np.array_equal(s_ids.numpy(), want_ids) and np.array_equal(
            s_sc.numpy().view(np.uint32), want_sc.view(np.uint32))
    if rank == 0:
        Path(result_dir, "ok").write_text("1" if ok else "0")
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_sharded_ivf_search_equals_unsharded_with_gloo_ranks(tmp_path, world):
    """world_size 2 and 4 on CPU: posting lists dealt by bytes, every rank
    probes all centroids and scans its own lists (the oracle stands in for
    the device search), all-gather, merge == the IVF top-k of the whole
    index, centered and not; and the same with the probe split by query
    slices (ivf_sharded_search: probe slice, all-gather of the lists, packed
    all-to-all and slice merges; 15 queries make uneven slices at world 4)
    on every rank."""
    import socket

    import torch.multiprocessing as mp

    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    mp.start_processes(_gloo_ivf_worker, args=(world, port, str(tmp_path)), nprocs=world,
                       join=True, start_method="spawn")
    assert (tmp_path / "ok").read_text() == "1"


def test_bench_generator_shapes_and_centering():
    import sys

    sys.path.insert(0, str(REPO))
    import bench

    base, query = bench.make_data(5000, 50)
    assert base.shape == (5000, 128) and query.shape == (50, 128)
    assert abs(float(base.mean(0, dtype=np.float64).max())) < 1e-3
    # the raw zeros (about 40%) become each column's minimum after centering
    zeros = np.mean(base == base.min(0, keepdims=True))
    assert 0.35 < zeros < 0.45
