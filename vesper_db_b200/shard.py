"""Multi-GPU sharding of an IVF-PQ database (one process per GPU).

The base set is split by vector: base chunk c belongs to rank c mod world.  Every
rank holds the same model (trained from the same sample with the same seeds, so
every rank probes the same lists), searches every query over its own shard, and the
per-rank top-k are merged after an all_gather.  Merging keeps, per query, the k best
by (distance, rank, position in the rank's result) -- the same candidates a single
index over the whole base would return, up to ties at the k-th distance.

`merge_topk` is the exchange step (NCCL on GPUs, gloo in the CPU tests);
`shard_of` / `chunks_of` are the partition rule.
"""
from __future__ import annotations


def chunks_of(rank: int, world: int, n_chunks: int) -> list[int]:
    """Base chunks held by `rank` (chunk c -> rank c mod world)."""
    return [c for c in range(n_chunks) if c % world == rank]


def merge_topk(dist, ids, k: int, group=None):
    """All-gather the per-rank [nq, k] (dist, ids) and keep the k smallest per query.

    Ties keep the lower rank, then the earlier position (a stable sort of the
    concatenation in rank order)."""
    import torch
    import torch.distributed as dist_mod

    world = dist_mod.get_world_size(group)
    gd = [torch.empty_like(dist) for _ in range(world)]
    gi = [torch.empty_like(ids) for _ in range(world)]
    dist_mod.all_gather(gd, dist.contiguous(), group=group)
    dist_mod.all_gather(gi, ids.contiguous(), group=group)
    cd = torch.cat(gd, 1)
    ci = torch.cat(gi, 1)
    order = torch.argsort(cd, dim=1, stable=True)[:, :k]
    return torch.gather(cd, 1, order), torch.gather(ci, 1, order)
