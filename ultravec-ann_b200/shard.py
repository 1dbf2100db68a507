"""Host-side sharding across ranks (one process per GPU).

Flat index: the base rows are split into contiguous ranges; every rank
encodes and scans its own range (records keep their global row ids).  IVF
index: the posting lists are dealt to ranks so that each rank holds about the
same number of record bytes; every rank keeps all centroids, probes
redundantly, and scans only the probed lists it owns, so each probed list is
scanned exactly once.  Either way the per-rank top-k lists are combined by
one all-gather and a merge.  The merge is a function argument so that the
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
