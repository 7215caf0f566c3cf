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
                  group=None, mode: int = 0, local=None, times: dict | None = None):
    """Search the whole batch over this rank's shard with the coarse stage split across
    ranks: rank r probes rows [r nq/W, (r+1) nq/W) (index.probe_device), the probe lists
    and distances are all-gathered, then index.search_batch_device_probed runs on the
    full batch.  queries [nq, dim] float32 and the outputs are tensors on the index's
    device; nq must be a multiple of the world size.  `bufs` caches the probe buffers
    between calls.

    local: this rank's rows of the batch, already on the device, when `queries` does not
    hold the batch yet (a batch that arrives from the host: each rank copies only its
    slice); the slices are all-gathered into `queries` after the probe.
    times: if given, host-side milliseconds of the three phases are added to
    times["probe_ms"], times["exchange_ms"] and times["search_ms"]."""
    import time

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
    if local is not None and tuple(local.shape) != (per, queries.shape[1]):
        raise ValueError("probed_search: `local` must hold this rank's nq / world rows")
    t0 = time.perf_counter()
    mine_q = local if local is not None else queries[rank * per:]
    index.probe_device(mine_q.data_ptr(), per, nprobe, mine.data_ptr(), mine_d.data_ptr())
    t1 = time.perf_counter()
    if local is not None:
        dist_mod.all_gather_into_tensor(queries, local, group=group)
    dist_mod.all_gather_into_tensor(probe, mine, group=group)
    dist_mod.all_gather_into_tensor(probe_d, mine_d, group=group)
    # The library runs on its own stream and does not order itself after the caller's:
    # the gathered lists must be complete before the search starts.
    if probe.is_cuda:
        torch.cuda.current_stream(probe.device).synchronize()
    t2 = time.perf_counter()
    index.search_batch_device_probed(queries.data_ptr(), nq, k, nprobe, probe.data_ptr(), probe_d.data_ptr(),
                                     out_ids.data_ptr(), out_d.data_ptr(), out_n.data_ptr(), mode=mode)
    if times is not None:
        t3 = time.perf_counter()
        for key2, v in (("probe_ms", t1 - t0), ("exchange_ms", t2 - t1), ("search_ms", t3 - t2)):
            times[key2] = times.get(key2, 0.0) + v * 1e3


class _DeviceArray:
    """A float32 vector at a raw device address, for torch.as_tensor (CUDA array
    interface, no copy)."""

    def __init__(self, ptr: int, n: int):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": "<f4", "data": (ptr, False), "version": 2}


class ThresholdExchange:
    """The threshold exchange of a sharded database (vesper_ivfpq_set_threshold_exchange)
    over torch.distributed: every rank's index hands its per-query upper bounds of the
    k-th distance to `__call__`, which replaces them with the minimum over the ranks (an
    all-reduce MIN issued on the index's stream, so no host wait).  Install on every
    rank's index with `install`, before the first search; every rank must then search
    the same batches with the same parameters, as the sharded search does anyway.

    `view(ptr, n)` makes the tensor over the library's buffer (a CUDA view by default;
    the CPU tests pass a host view)."""

    def __init__(self, group=None, view=None):
        self.group = group
        self.view = view
        self.error = None
        self.calls = 0

    def __call__(self, d_tau, n, stream, user) -> int:
        try:
            import torch
            import torch.distributed as dist_mod
            if self.view is not None:
                t = self.view(d_tau, n)
            else:
                t = torch.as_tensor(_DeviceArray(d_tau, n), device=torch.device("cuda", torch.cuda.current_device()))
            if t.is_cuda:
                with torch.cuda.stream(torch.cuda.ExternalStream(stream, device=t.device)):
                    dist_mod.all_reduce(t, op=dist_mod.ReduceOp.MIN, group=self.group)
            else:
                dist_mod.all_reduce(t, op=dist_mod.ReduceOp.MIN, group=self.group)
            self.calls += 1
            return 0
        except Exception as e:  # reported to the library as a failed exchange
            self.error = e
            return 1

    def install(self, index, split: bool = True):
        """split: each rank runs the threshold pass for 1/world of the batch (queries q
        with q % world == rank) and takes the others' bounds from the exchange."""
        import torch.distributed as dist_mod
        if split and dist_mod.is_initialized():
            index.set_threshold_exchange(self, dist_mod.get_rank(self.group), dist_mod.get_world_size(self.group))
        else:
            index.set_threshold_exchange(self)
        return self


class ShardResults:
    """Per-rank result buffers of a sharded search, packed so that one all-gather moves
    them, and the device merge (vesper_topk_merge_device) of the gathered parts.

    `ids` int64 [nq, k], `dist` float32 [nq, k] and `counts` int32 [nq] are views into one
    int32 buffer; the library's search writes them.  `merge()` all-gathers the buffer
    over the group and merges the parts on the current CUDA stream, returning
    (dist [nq, k], ids [nq, k], counts [nq]) of the whole database."""

    def __init__(self, nq: int, k: int, device, group=None, world: int | None = None):
        import torch
        import torch.distributed as dist_mod
        self.nq, self.k, self.group = nq, k, group
        self.world = world if world is not None else dist_mod.get_world_size(group)
        nk = nq * k
        off_ids = nk + (nk & 1)              # int64 view needs an 8-byte aligned offset
        off_n = off_ids + 2 * nk
        words = off_n + nq
        words += words & 1                   # each part starts 8-byte aligned
        self.words, self.off_ids, self.off_n = words, off_ids, off_n
        self.buf = torch.zeros(words, dtype=torch.int32, device=device)
        self.dist = self.buf[:nk].view(torch.float32).view(nq, k)
        self.ids = self.buf[off_ids:off_ids + 2 * nk].view(torch.int64).view(nq, k)
        self.counts = self.buf[off_n:off_n + nq]
        self.gathered = torch.empty(self.world * words, dtype=torch.int32, device=device)
        self.out_ids = torch.empty((nq, k), dtype=torch.int64, device=device)
        self.out_d = torch.empty((nq, k), dtype=torch.float32, device=device)
        self.out_n = torch.empty(nq, dtype=torch.int32, device=device)

    def parts_layout(self):
        """Where part p's arrays sit in the gathered buffer: (byte offset of its first
        element from the buffer's start, stride between parts in elements of that array)
        for the distances (float32), ids (int64) and counts (int32) -- the arguments of
        vesper_topk_merge_device."""
        return {"dist": (0, self.words), "ids": (4 * self.off_ids, self.words // 2),
                "counts": (4 * self.off_n, self.words)}

    def merge(self):
        import torch
        import torch.distributed as dist_mod

        from . import _native as N
        from .index import _check
        dist_mod.all_gather_into_tensor(self.gathered, self.buf, group=self.group)
        g = self.gathered.data_ptr()
        lay = self.parts_layout()
        lib = N.load()
        _check(lib, lib.vesper_topk_merge_device(
            self.world, self.nq, self.k, g + lay["dist"][0], lay["dist"][1], g + lay["ids"][0], lay["ids"][1],
            g + lay["counts"][0], lay["counts"][1], self.out_ids.data_ptr(), self.out_d.data_ptr(),
            self.out_n.data_ptr(), torch.cuda.current_stream(self.buf.device).cuda_stream))
        return self.out_d, self.out_ids, self.out_n


# ------------------------------------------------------------------ sharded k-means
class KmeansPPSampler:
    """The k-means++ draws of kmeans_plusplus_init (src/index/kmeans.cpp:45-89) for n
    points (vesper_kmeanspp_sampler_*): `first` is the first row; `next(d2)` takes the
    D^2 value of every point (float32, point order) and returns the next row."""

    def __init__(self, seed: int, n: int):
        import ctypes as C

        from . import _native as N
        from .index import _check
        self._lib = N.load()
        self._h = C.c_void_p()
        first = C.c_size_t(0)
        _check(self._lib, self._lib.vesper_kmeanspp_sampler_create(seed, n, C.byref(self._h), C.byref(first)))
        self.first = int(first.value)
        self.n = n

    def next(self, d2) -> int:
        import ctypes as C

        import numpy as np

        from .index import _check
        h = np.ascontiguousarray(d2, dtype=np.float32)
        if h.shape != (self.n,):
            raise ValueError("KmeansPPSampler.next: d2 must hold one value per point")
        idx = C.c_size_t(0)
        _check(self._lib, self._lib.vesper_kmeanspp_sampler_next(
            self._h, h.ctypes.data_as(C.POINTER(C.c_float)), C.byref(idx)))
        return int(idx.value)

    def close(self):
        if self._h:
            self._lib.vesper_kmeanspp_sampler_destroy(self._h)
            self._h = None

    def __del__(self):
        self.close()


class GpuKmeansOps:
    """The per-shard k-means steps on this process's current GPU
    (vesper_kmeans_shard_* in libvesper_c.so).  Tensors are CUDA tensors; assignments
    are int32 tensors holding the uint32 cluster ids, counts int64 holding uint64."""

    def __init__(self):
        import ctypes as C

        from . import _native as N
        from .index import _check
        self._lib = N.load()
        self._h = C.c_void_p()
        _check(self._lib, self._lib.vesper_kmeans_shard_create(C.byref(self._h)))

    @staticmethod
    def _ready(t):
        # the library runs on its own stream: finish what torch queued on the inputs
        import torch
        if t.is_cuda:
            torch.cuda.current_stream(t.device).synchronize()

    def _call(self, fn, *args):
        from .index import _check
        _check(self._lib, getattr(self._lib, fn)(self._h, *args))

    def assign(self, x, c, keep, a, mind):
        self._ready(x)
        self._call("vesper_kmeans_shard_assign", x.data_ptr(), x.shape[0], x.shape[1], c.data_ptr(), c.shape[0],
                   int(bool(keep)), a.data_ptr(), mind.data_ptr())

    def pp_update(self, x, crow, mind):
        self._ready(x)
        self._call("vesper_kmeans_shard_pp_update", x.data_ptr(), x.shape[0], x.shape[1], crow.data_ptr(),
                   mind.data_ptr())

    def accumulate(self, x, a, k, algorithm, s, comp, count):
        self._ready(x)
        self._call("vesper_kmeans_shard_accumulate", x.data_ptr(), x.shape[0], x.shape[1], a.data_ptr(), k,
                   algorithm, s.data_ptr(), comp.data_ptr(), count.data_ptr())

    def finish(self, s, count, algorithm, c):
        self._ready(s)
        self._call("vesper_kmeans_shard_finish", s.data_ptr(), count.data_ptr(), c.shape[0], c.shape[1], algorithm,
                   c.data_ptr())

    def running_inertia(self, x, c, a, total: float) -> float:
        import ctypes as C
        self._ready(x)
        t = C.c_float(total)
        self._call("vesper_kmeans_shard_running_inertia", x.data_ptr(), x.shape[0], x.shape[1], c.data_ptr(),
                   a.data_ptr(), C.byref(t))
        return t.value

    @staticmethod
    def sampler(seed: int, n: int):
        return KmeansPPSampler(seed, n)

    def close(self):
        if self._h:
            self._lib.vesper_kmeans_shard_destroy(self._h)
            self._h = None

    def __del__(self):
        self.close()


def kmeans_fit_sharded(shards, k: int, max_iter: int = 25, epsilon: float = 1e-4, seed: int = 42,
                       algorithm: int = 0, group=None, ops=None):
    """k-means over points sharded across processes (one per GPU), equal bit for bit to
    the one-GPU fit (vesper_kmeans_fit_device) over the concatenation of every rank's
    shards in rank order.

    `shards`: this rank's [n_i, dim] float32 tensors, in point order (several per rank
    are allowed).  algorithm 0 = Elkan (KmeansElkan::cluster,
    src/index/kmeans_elkan.cpp:293-430), 1 = Lloyd (kmeans_cluster, src/index/kmeans.cpp:
    137-252, one run).  Centroids are replicated; per iteration each rank assigns its own
    points, the per-point distances are all-gathered for the fp64 inertia in point order,
    and the mean update is a chain in rank order (each rank continues the per-cluster
    running sums the previous rank sent it, the last rank finishes the means and
    broadcasts them), which keeps the reference's point-order sums exact.  k-means++
    gathers the D^2 vector per centroid and draws on every rank with the same sampler.
    Lloyd's final inertia, a float running total over every term, travels the same chain.

    Returns (centroids [k, dim] tensor, [assignments per shard], iterations, inertia)."""
    import numpy as np
    import torch
    import torch.distributed as dist

    if ops is None:
        ops = GpuKmeansOps()
    on = dist.is_available() and dist.is_initialized()
    world = dist.get_world_size(group) if on else 1
    rank = dist.get_rank(group) if on else 0
    dev = shards[0].device
    d = int(shards[0].shape[1])
    n_local = sum(int(s.shape[0]) for s in shards)
    if world > 1:
        t = torch.tensor([n_local], dtype=torch.int64, device=dev)
        allt = [torch.empty_like(t) for _ in range(world)]
        dist.all_gather(allt, t, group=group)
        rank_n = [int(v.item()) for v in allt]
    else:
        rank_n = [n_local]
    n = sum(rank_n)
    if k == 0:
        raise ValueError("k must be > 0")
    if n < k:
        raise ValueError("Not enough data points for k clusters")
    base = sum(rank_n[:rank])
    elkan = algorithm == 0

    def src(r):
        return dist.get_global_rank(group, r) if group is not None else r

    def gather_host(parts):
        local = torch.cat(parts) if len(parts) > 1 else parts[0]
        if world == 1:
            return local.cpu().numpy()
        m = max(rank_n)
        buf = torch.zeros(m, dtype=local.dtype, device=dev)
        buf[:n_local] = local
        out = torch.empty(world * m, dtype=local.dtype, device=dev)
        dist.all_gather_into_tensor(out, buf, group=group)
        h = out.cpu().numpy()
        return np.concatenate([h[r * m:r * m + rank_n[r]] for r in range(world)])

    def fetch_row(gidx, row):
        owner = int(np.searchsorted(np.cumsum(rank_n), gidx, side="right"))
        if owner == rank:
            i = gidx - base
            for s in shards:
                if i < s.shape[0]:
                    row.copy_(s[i])
                    break
                i -= s.shape[0]
        if world > 1:
            dist.broadcast(row, src=src(owner), group=group)

    # k-means++ (kmeans.cpp:45-89)
    cent = torch.empty((k, d), dtype=torch.float32, device=dev)
    sampler = ops.sampler(seed, n)
    fetch_row(sampler.first, cent[0])
    mind = [torch.full((s.shape[0],), float(np.finfo(np.float32).max), dtype=torch.float32, device=dev)
            for s in shards]
    for c in range(1, k):
        for s, md in zip(shards, mind):
            ops.pp_update(s, cent[c - 1], md)
        fetch_row(sampler.next(gather_host(mind)), cent[c])
    sampler.close()

    asg = [torch.zeros(s.shape[0], dtype=torch.int32, device=dev) for s in shards]
    dst = [torch.empty(s.shape[0], dtype=torch.float32, device=dev) for s in shards]

    def estep(keep):
        for s, a, md in zip(shards, asg, dst):
            ops.assign(s, cent, keep, a, md)

    def inertia():
        h = gather_host(dst).astype(np.float64)
        return np.float32(np.cumsum(h)[-1]) if h.size else np.float32(0.0)

    def mstep():
        sm = torch.zeros((k, d), dtype=torch.float64, device=dev)
        comp = torch.zeros((k, d), dtype=torch.float64, device=dev)
        cnt = torch.zeros(k, dtype=torch.int64, device=dev)
        if world > 1 and rank > 0:
            for t_ in (sm, comp, cnt):
                dist.recv(t_, src=src(rank - 1), group=group)
        for s, a in zip(shards, asg):
            ops.accumulate(s, a, k, algorithm, sm, comp, cnt)
        if rank < world - 1:
            for t_ in (sm, comp, cnt):
                dist.send(t_, dst=src(rank + 1), group=group)
        else:
            ops.finish(sm, cnt, algorithm, cent)
        if world > 1:
            dist.broadcast(cent, src=src(world - 1), group=group)

    eps = np.float32(epsilon)
    tiny = np.float32(1e-10)
    prev = np.float32(np.finfo(np.float32).max)
    if elkan:
        estep(False)
    it = 0
    while it < max_iter:
        if not elkan or it > 0:
            estep(elkan)
        cur = inertia()
        change = np.float32(abs(np.float32(prev - cur))) / np.float32(prev + tiny)
        if change < eps:
            break
        prev = cur
        mstep()
        it += 1
    if elkan:
        result_inertia = float(prev)
    else:
        # kmeans.cpp:230-241: one float running total over every term, in point order,
        # passed along the ranks like the mean-update state
        mstep()
        tot = torch.zeros(1, dtype=torch.float32, device=dev)
        if world > 1 and rank > 0:
            dist.recv(tot, src=src(rank - 1), group=group)
        run = float(tot.item())
        for s, a in zip(shards, asg):
            run = ops.running_inertia(s, cent, a, run)
        tot.fill_(run)
        if rank < world - 1:
            dist.send(tot, dst=src(rank + 1), group=group)
        if world > 1:
            dist.broadcast(tot, src=src(world - 1), group=group)
        result_inertia = float(tot.item())
    return cent, asg, it, result_inertia
