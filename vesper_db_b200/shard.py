"""Multi-GPU sharding of an IVF-PQ database (one process per GPU).

The base set is split by vector: base chunk c belongs to rank c mod world.  Every
rank holds the same model (trained from the same sample with the same seeds, so
every rank probes the same lists), searches every query over its own shard, and the
per-rank top-k are merged after an all_gather.  Merging keeps, per query, the k best
by (distance, rank, position in the rank's result) -- the same candidates a single
index over the whole base would return, up to ties at the k-th distance.

`merge_topk` is the exchange step (NCCL on GPUs, gloo in the CPU tests);
`chunks_of` is the partition rule.  `probed_search` splits the coarse stage, which is
the same on every shard: each rank probes 1/world of the batch and the probe lists are
all-gathered before every rank searches the whole batch over its shard.
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


def probed_search(index, queries, k: int, nprobe: int, nlist: int, out_ids, out_d, out_n, bufs: dict,
                  group=None, mode: int = 0):
    """Search the whole batch over this rank's shard with the coarse stage split across
    ranks: rank r probes rows [r nq/W, (r+1) nq/W) (index.probe_device), the probe lists
    and distances are all-gathered, then index.search_batch_device_probed runs on the
    full batch.  queries [nq, dim] float32 and the outputs are tensors on the index's
    device; nq must be a multiple of the world size.  `bufs` caches the probe buffers
    between calls."""
    import torch
    import torch.distributed as dist_mod

    world = dist_mod.get_world_size(group)
    rank = dist_mod.get_rank(group)
    nq = queries.shape[0]
    if nq % world:
        raise ValueError("probed_search: the batch must split evenly across the ranks")
    npq = min(nprobe, nlist)
    key = (nq, npq)
    if key not in bufs:
        dev = queries.device
        bufs[key] = (torch.empty((nq, npq), dtype=torch.int32, device=dev),
                     torch.empty((nq, npq), dtype=torch.float32, device=dev),
                     torch.empty((nq // world, npq), dtype=torch.int32, device=dev),
                     torch.empty((nq // world, npq), dtype=torch.float32, device=dev))
    probe, probe_d, mine, mine_d = bufs[key]
    per = nq // world
    index.probe_device(queries[rank * per:].data_ptr(), per, nprobe, mine.data_ptr(), mine_d.data_ptr())
    dist_mod.all_gather_into_tensor(probe, mine, group=group)
    dist_mod.all_gather_into_tensor(probe_d, mine_d, group=group)
    # The library runs on its own stream and does not order itself after the caller's:
    # the gathered lists must be complete before the search starts.
    if probe.is_cuda:
        torch.cuda.current_stream(probe.device).synchronize()
    index.search_batch_device_probed(queries.data_ptr(), nq, k, nprobe, probe.data_ptr(), probe_d.data_ptr(),
                                     out_ids.data_ptr(), out_d.data_ptr(), out_n.data_ptr(), mode=mode)
