"""Sharded k-means (vesper_db_b200.shard.kmeans_fit_sharded) on CPU, gloo, world size 2.

The per-shard steps run in an oracle-backed stand-in for the GPU (the same arithmetic:
reference-order distances, lowest index or keep-on-tie argmin, Kahan or plain fp64
running sums in point order), while the driver's collectives -- the gathered D^2 and
distance vectors, the row broadcasts, the rank-order chain of the mean update and the
centroid broadcast -- run over gloo.  Rank 0 holds two shards and rank 1 one, of
unequal sizes.  The result must equal the reference's own k-means on the whole set
(tests/golden/kmeans_small.npz) bit for bit.
"""
import os
import socket

import numpy as np
import pytest

from conftest import GOLDEN, ROOT

SPLITS = [(0, 1000), (1000, 1500), (1500, 3000)]   # rank 0: first two, rank 1: last
OWNER = [0, 0, 1]


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


class OracleKmeansOps:
    """The shard steps on CPU tensors, in the reference's arithmetic (the oracle)."""

    def __init__(self, oracle):
        self.o = oracle

    def assign(self, x, c, keep, a, mind):
        xn, cn = x.numpy(), c.numpy()
        best = self.o.assign(xn, cn)
        dmin = np.array([self.o.l2_sq(xn[i], cn[best[i]]) for i in range(xn.shape[0])], np.float32)
        if keep:
            cur = a.numpy().view(np.uint32)
            dcur = np.array([self.o.l2_sq(xn[i], cn[cur[i]]) for i in range(xn.shape[0])], np.float32)
            best = np.where(dcur == dmin, cur, best)
        a.numpy().view(np.uint32)[:] = best
        mind.numpy()[:] = dmin

    def pp_update(self, x, crow, mind):
        xn, c = x.numpy(), crow.numpy()
        d = np.array([self.o.l2_sq(xn[i], c) for i in range(xn.shape[0])], np.float32)
        m = mind.numpy()
        m[:] = np.where(d < m, d, m)

    def accumulate(self, x, a, k, algorithm, s, comp, count):
        xn, an = x.numpy(), a.numpy().view(np.uint32)
        sn, cn, cnt = s.numpy(), comp.numpy(), count.numpy()
        for i in range(xn.shape[0]):
            c = an[i]
            v = xn[i].astype(np.float64)
            cnt[c] += 1
            if algorithm == 0:
                y = v - cn[c]
                t = sn[c] + y
                cn[c] = (t - sn[c]) - y
                sn[c] = t
            else:
                sn[c] = sn[c] + v

    def finish(self, s, count, algorithm, c):
        sn, cnt, cn = s.numpy(), count.numpy(), c.numpy()
        for j in range(cn.shape[0]):
            if cnt[j]:
                cn[j] = (sn[j] * (1.0 / float(cnt[j]))) if algorithm == 0 else (sn[j] / float(cnt[j]))

    def running_inertia(self, x, c, a, total):
        xn, cn, an = x.numpy(), c.numpy(), a.numpy().view(np.uint32)
        t = np.float32(total)
        for i in range(xn.shape[0]):
            diff = xn[i] - cn[an[i]]
            for v in diff * diff:
                t = np.float32(t + v)
        return float(t)

    @staticmethod
    def sampler(seed, n):
        from vesper_db_b200.shard import KmeansPPSampler
        return KmeansPPSampler(seed, n)


def _worker(rank, world, port, algorithm, k, iters, eps, out_path):
    import sys
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import torch
    import torch.distributed as dist
    from oracle_lib import Oracle

    from vesper_db_b200.shard import kmeans_fit_sharded
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        x = np.load(os.path.join(GOLDEN, "kmeans_small.npz"))["x"]
        shards = [torch.from_numpy(x[a:b].copy()) for (a, b), o in zip(SPLITS, OWNER) if o == rank]
        c, asg, it, inertia = kmeans_fit_sharded(shards, k, iters, eps, 42, algorithm,
                                                 ops=OracleKmeansOps(Oracle()))
        a = torch.cat(asg)
        parts = [torch.zeros(1500, dtype=torch.int32) for _ in range(world)]
        dist.all_gather(parts, a)
        if rank == 0:
            np.savez(out_path, c=c.numpy(), a=torch.cat(parts).numpy().view(np.uint32), it=it, inertia=inertia)
        dist.barrier()
    finally:
        dist.destroy_process_group()


def _run(tmp_path, algorithm, k, iters, eps):
    import torch.multiprocessing as mp
    out = str(tmp_path / "km.npz")
    mp.start_processes(_worker, args=(2, _free_port(), algorithm, k, iters, eps, out), nprocs=2, join=True,
                       start_method="spawn")
    return np.load(out)


def test_sharded_elkan_equals_reference(tmp_path):
    g = np.load(os.path.join(GOLDEN, "kmeans_small.npz"))
    r = _run(tmp_path, 0, 48, 25, 1e-4)
    assert np.array_equal(r["c"], g["elkan_c"])
    assert np.array_equal(r["a"], g["elkan_a"])
    assert int(r["it"]) == int(g["elkan_it"]) and np.float32(r["inertia"]) == np.float32(g["elkan_inertia"])


def test_sharded_lloyd_equals_reference(tmp_path):
    g = np.load(os.path.join(GOLDEN, "kmeans_small.npz"))
    r = _run(tmp_path, 1, 48, 20, 0.0)
    assert np.array_equal(r["c"], g["lloyd_c"])
    assert np.array_equal(r["a"], g["lloyd_a"])
    assert int(r["it"]) == int(g["lloyd_it"])
    assert np.float32(r["inertia"]) == np.float32(g["lloyd_inertia"])


def test_sampler_reproduces_reference_kmeanspp(oracle):
    """The C-ABI sampler with the oracle's D^2 updates picks the reference's rows."""
    from vesper_db_b200.shard import KmeansPPSampler
    g = np.load(os.path.join(GOLDEN, "kmeans_small.npz"))
    x = g["x"]
    s = KmeansPPSampler(42, x.shape[0])
    rows = [s.first]
    mind = np.full(x.shape[0], np.finfo(np.float32).max, np.float32)
    for _ in range(1, 48):
        d = np.array([oracle.l2_sq(x[i], x[rows[-1]]) for i in range(x.shape[0])], np.float32)
        mind = np.where(d < mind, d, mind)
        rows.append(s.next(mind))
    assert np.array_equal(x[rows], g["kpp"])
