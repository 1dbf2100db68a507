"""Host-side sharding across ranks (one process per GPU).

Flat index: the base rows are split into contiguous ranges; every rank
encodes and scans its own range (records keep their global row ids).  IVF
index: the posting lists are dealt to ranks so that each rank holds about the
same number of record bytes; every rank keeps all centroids, probes its own
query slice, shares the probe lists by one all-gather, and scans only the
probed lists it owns, so each query is probed once and each probed list is
scanned once (ivf_sharded_search).  The flat search exchanges first-pass
bounds between the shards before they keep candidates (sharded_search).
Both combine the per-rank lists with one packed all-to-all of query slices,
per-slice merges and one all-gather (combine_topk); gather_topk is the plain
all-gather + merge.  The merge is a function argument so that the
same sequence runs with the device merge (`uv_topk_merge`) under NCCL and
with a host merge under gloo.
"""
from __future__ import annotations


def shard_range(n: int, rank: int, world: int) -> tuple[int, int]:
    """Rows [lo, hi) owned by `rank`: contiguous, sizes differing by <= 1."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("bad rank/world")
    return rank * n // world, (rank + 1) * n // world


def ivf_list_owners(list_sizes, world: int):
    """Owner rank of every posting list, balancing record bytes: lists in
    descending size (ties by list number) each go to the rank holding the
    fewest records so far (ties by lower rank).  Deterministic, so every rank
    computes the same map from the same sizes."""
    import numpy as np

    if world < 1:
        raise ValueError("bad world size")
    sizes = np.asarray(list_sizes, np.int64)
    order = np.lexsort((np.arange(len(sizes)), -sizes))
    load = np.zeros(world, np.int64)
    owner = np.empty(len(sizes), np.int32)
    for l in order:
        r = int(np.argmin(load))
        owner[l] = r
        load[r] += sizes[l]
    return owner


def ivf_owned_rows(assign, owners, rank: int):
    """Row numbers (ascending) whose posting list `rank` owns."""
    import numpy as np

    assign = np.asarray(assign)
    return np.nonzero(np.asarray(owners)[assign] == rank)[0]


def gather_topk(local_ids, local_scores, k: int, dist, merge):
    """All-gather every rank's (nq, k) top-k and merge to the global top-k.

    `dist` is torch.distributed with an initialized group; `merge(ids, scores,
    k)` takes (nq, world, k_in) arrays sorted by (score desc, id asc) and
    returns the (nq, k) merge.  With world == 1 the local lists are returned.
    """
    import torch

    world = dist.get_world_size()
    if world == 1:
        return local_ids, local_scores
    nq, kin = local_ids.shape
    # concatenated along dim 0 (the layout every backend accepts), then
    # viewed as (world, nq, k_in) and transposed to (nq, world, k_in)
    g_ids = torch.empty((world * nq, kin), dtype=local_ids.dtype, device=local_ids.device)
    g_sc = torch.empty((world * nq, kin), dtype=local_scores.dtype, device=local_scores.device)
    dist.all_gather_into_tensor(g_ids, local_ids.contiguous())
    dist.all_gather_into_tensor(g_sc, local_scores.contiguous())
    g_ids = g_ids.view(world, nq, kin).permute(1, 0, 2).contiguous()
    g_sc = g_sc.view(world, nq, kin).permute(1, 0, 2).contiguous()
    return merge(g_ids, g_sc, k)


def query_slice(nq: int, rank: int, world: int) -> tuple[int, int]:
    """Queries [lo, hi) whose merge `rank` does: contiguous slices."""
    return rank * nq // world, (rank + 1) * nq // world


def sharded_search(begin, k: int, dist, pack, unpack, merge_packed, deferred: bool = False):
    """The flat search of a base split across ranks (one index shard each,
    global ids), as uv_index_search_begin / set_bounds / finish plus the
    merge describe it:

    1. `begin(world)` starts the shard's search and exposes its (nq, m)
       best first-pass lower bounds; one all-gather makes them (world * nq,
       m), shard-major, on every rank, and every shard takes the k-th largest
       of their union as its threshold (`set_bounds`).
    2. `finish()` gives the shard's lists: only records that can be in the
       global top k survive the shared threshold.  With `deferred`, finish
       queues that work without waiting for the device, and after the
       combine `check()` on every rank and one all-reduce tell whether any
       shard rescanned an overflowed query exactly, in which case the
       (rewritten) lists are combined again.
    3. The lists travel once, packed (ids and scores in one 12-byte record,
       `pack`): an all-to-all hands rank r every shard's lists for its query
       slice, rank r merges its slice over the shards (`merge_packed` with
       row stride k and list stride rows * k), and one all-gather of the
       merged, packed slices (padded to the largest slice) gives every rank
       the (nq, k) answer.

    Every rank takes the same collective steps in the same order.  `pack`,
    `unpack` and `merge_packed` are the device routines under NCCL and host
    stand-ins under gloo."""
    import torch

    world = dist.get_world_size()
    s = begin(world)
    try:
        bounds = s.bounds
        nq, m = bounds.shape
        gathered = torch.empty((world * nq, m), dtype=bounds.dtype, device=bounds.device)
        dist.all_gather_into_tensor(gathered, bounds.contiguous())
        s.set_bounds(gathered, world)
        if deferred:
            # queued without waiting for the device; the combine's
            # collectives follow at once, the outcome check after them
            ids, scores = s.finish(deferred=True)
            out = combine_topk(ids, scores, k, dist, pack, unpack, merge_packed)
            over = torch.tensor([1 if s.check() else 0], dtype=torch.int32,
                                device=bounds.device)
            dist.all_reduce(over, op=dist.ReduceOp.MAX)
            if int(over.item()):
                # a shard rescanned overflowed queries exactly: merge again
                out = combine_topk(ids, scores, k, dist, pack, unpack, merge_packed)
        else:
            ids, scores = s.finish()
            out = combine_topk(ids, scores, k, dist, pack, unpack, merge_packed)
    finally:
        s.close()
    return out


def combine_topk(ids, scores, k: int, dist, pack, unpack, merge_packed):
    """Every rank's (nq, k) lists -> the global (nq, k) top-k on every rank:
    the lists travel once, packed (`pack`: ids and scores in one 12-byte
    record); an all-to-all hands rank r every shard's lists for its query
    slice, rank r merges its slice (`merge_packed`, row stride k, list stride
    rows * k), and one all-gather of the merged, packed slices (padded to the
    largest slice) gives every rank the answer."""
    import torch

    world = dist.get_world_size()
    rank = dist.get_rank()
    nq = ids.shape[0]
    packed = pack(ids, scores).reshape(-1)
    lo, hi = query_slice(nq, rank, world)
    rows = hi - lo
    in_splits = [(query_slice(nq, r, world)[1] - query_slice(nq, r, world)[0]) * k * 3
                 for r in range(world)]
    recv = torch.empty(world * rows * k * 3, dtype=packed.dtype, device=packed.device)
    dist.all_to_all_single(recv, packed, [rows * k * 3] * world, in_splits)
    m_ids, m_sc = merge_packed(recv, rows, world, k, k, k, rows * k)
    rows_max = (nq + world - 1) // world
    if rows == rows_max:
        mine = pack(m_ids, m_sc).reshape(rows, k, 3)
    else:
        mine = torch.zeros((rows_max, k, 3), dtype=packed.dtype, device=packed.device)
        if rows > 0:
            mine[:rows] = pack(m_ids, m_sc).reshape(rows, k, 3)
    allp = torch.empty((world * rows_max, k, 3), dtype=packed.dtype, device=packed.device)
    dist.all_gather_into_tensor(allp, mine)
    if rows_max * world == nq:
        return unpack(allp)  # equal slices: the gathered rows are the queries in order
    allp = allp.view(world, rows_max, k, 3)
    parts = [allp[r, :query_slice(nq, r, world)[1] - query_slice(nq, r, world)[0]]
             for r in range(world)]
    return unpack(torch.cat(parts, 0))


def ivf_sharded_search(ivf, queries, k: int, nprobe: int, dist, pack, unpack, merge_packed):
    """The IVF search of a base whose posting lists are dealt to ranks
    (ivf_list_owners): rank r probes only its query slice (every rank holds
    all centroids), one all-gather shares the probe lists, every rank scans
    the probed lists it holds for all queries (IvfIndex.search_lists; lists
    held elsewhere are skipped), and the per-rank lists combine as in
    combine_topk.  The probe is done once per query instead of once per
    rank."""
    import torch

    world = dist.get_world_size()
    rank = dist.get_rank()
    nq = queries.shape[0]
    lo, hi = query_slice(nq, rank, world)
    rows_max = (nq + world - 1) // world
    mine = ivf.probe(queries[lo:hi], nprobe)
    if not hasattr(mine, "device"):
        mine = torch.from_numpy(mine)
    pad = torch.full((rows_max, nprobe), -1, dtype=torch.int32, device=mine.device)
    pad[:hi - lo] = mine
    allp = torch.empty((world * rows_max, nprobe), dtype=torch.int32, device=mine.device)
    dist.all_gather_into_tensor(allp, pad)
    if rows_max * world == nq:
        lists = allp
    else:
        allp = allp.view(world, rows_max, nprobe)
        lists = torch.cat([allp[r, :query_slice(nq, r, world)[1] - query_slice(nq, r, world)[0]]
                           for r in range(world)], 0)
    ids, scores = ivf.search_lists(queries, k, lists)
    if not hasattr(ids, "device"):
        ids, scores = torch.from_numpy(ids), torch.from_numpy(scores)
    return combine_topk(ids, scores, k, dist, pack, unpack, merge_packed)


def pack_host(ids, scores):
    """Host stand-in of uv_topk_pack: (nq, k) -> (nq, k, 3) int32."""
    import numpy as np
    import torch

    i = np.ascontiguousarray(ids.cpu().numpy() if hasattr(ids, "cpu") else ids, np.int64)
    s = np.ascontiguousarray(scores.cpu().numpy() if hasattr(scores, "cpu") else scores,
                             np.float32)
    out = np.empty(i.shape + (3,), np.int32)
    out[..., 0] = (i & 0xFFFFFFFF).astype(np.uint32).view(np.int32)
    out[..., 1] = (i >> 32).astype(np.int64).astype(np.int32)
    out[..., 2] = s.view(np.int32)
    return torch.from_numpy(out)


def unpack_host(packed):
    """Host stand-in of the unpack: (..., 3) int32 -> ids, scores."""
    import torch

    lo = packed[..., 0].to(torch.int64) & 0xFFFFFFFF
    hi = packed[..., 1].to(torch.int64)
    return (hi << 32) | lo, packed[..., 2].contiguous().view(torch.float32)


def merge_packed_host(recv, rows: int, n_lists: int, k_in: int, k: int, row_stride: int,
                      list_stride: int):
    """Host stand-in of uv_topk_merge_packed with strides."""
    import numpy as np
    import torch

    p = recv.cpu().numpy().reshape(-1, 3)
    ids = np.empty((rows, n_lists, k_in), np.int64)
    sc = np.empty((rows, n_lists, k_in), np.float32)
    for q in range(rows):
        for l in range(n_lists):
            r = p[q * row_stride + l * list_stride:][:k_in]
            ids[q, l] = (r[:, 0].astype(np.int64) & 0xFFFFFFFF) | (r[:, 1].astype(np.int64) << 32)
            sc[q, l] = r[:, 2].view(np.float32)
    return merge_host(torch.from_numpy(ids), torch.from_numpy(sc), k)


def merge_host(ids, scores, k: int):
    """Reference merge on the host (numpy/torch CPU): score desc, id asc,
    NaN last, unfilled slots (id < 0) dropped and re-padded with (-1, -inf)."""
    import numpy as np

    ids_n = ids.cpu().numpy() if hasattr(ids, "cpu") else np.asarray(ids)
    sc_n = scores.cpu().numpy() if hasattr(scores, "cpu") else np.asarray(scores)
    nq = ids_n.shape[0]
    out_i = np.full((nq, k), -1, np.int64)
    out_s = np.full((nq, k), -np.inf, np.float32)
    for q in range(nq):
        cand = [(-(s if s == s else -np.inf), int(i), s)
                for i, s in zip(ids_n[q].ravel(), sc_n[q].ravel()) if i >= 0]
        cand.sort(key=lambda c: (c[0], c[1]))
        for j, (_, i, s) in enumerate(cand[:k]):
            out_i[q, j] = i
            out_s[q, j] = s
    if hasattr(ids, "cpu"):
        import torch

        return torch.from_numpy(out_i), torch.from_numpy(out_s)
    return out_i, out_s
