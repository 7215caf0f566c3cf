"""Multi-rank sharding logic on CPU (gloo, world size 2).

Each rank holds the base chunks c with c mod world == rank, searches all queries over
its shard (the oracle stands in for the per-GPU index), and the per-rank top-k are
merged with vesper_db_b200.shard.merge_topk.  The merged result must equal a single
search over the whole base (the reference's own results on its golden index), up to
ties at the k-th distance.
"""
import os
import socket

import numpy as np
import pytest

from conftest import GOLDEN, ROOT, assert_topk_equivalent, golden_case

CHUNK = 250


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, name, k, nprobe, out_path):
    import sys
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import torch
    import torch.distributed as dist
    from oracle_lib import Oracle

    from vesper_db_b200.shard import chunks_of, merge_topk
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        f, model, data = golden_case(name)
        base = data["base"]
        ids_all = np.arange(base.shape[0], dtype=np.uint64) * 3 + 7
        mine = chunks_of(rank, world, base.shape[0] // CHUNK)
        rows = np.concatenate([np.arange(c * CHUNK, (c + 1) * CHUNK) for c in mine])
        orc = Oracle()
        a, codes = orc.ivfpq_add(base[rows], model["centroids"], model["rotation"], model["codebooks"], model["m"])
        order = np.argsort(a, kind="stable")
        offs = np.zeros(model["nlist"] + 1, np.uint64)
        offs[1:] = np.cumsum(np.bincount(a, minlength=model["nlist"]))
        lid = ids_all[rows][order]
        q = data["queries"]
        rid, rd, rcnt = orc.ivfpq_search(q, model["centroids"], model["rotation"], model["codebooks"], model["m"],
                                         offs, lid, codes[order], k, nprobe)
        # empty result slots must never win the merge
        rd = np.where(np.arange(k)[None, :] < rcnt[:, None], rd, np.inf).astype(np.float32)
        md, mi = merge_topk(torch.from_numpy(rd), torch.from_numpy(rid.astype(np.int64)), k)
        if rank == 0:
            np.savez(out_path, d=md.numpy(), ids=mi.numpy().astype(np.uint64))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("name,k,nprobe", [("plain_d64_m8", 10, 4), ("opq_d32_m4", 100, 8)])
def test_sharded_merge_equals_single_index(tmp_path, name, k, nprobe):
    import torch.multiprocessing as mp
    out = str(tmp_path / "merged.npz")
    mp.start_processes(_worker, args=(2, _free_port(), name, k, nprobe, out), nprocs=2, join=True,
                       start_method="spawn")
    got = np.load(out)
    _, _, data = golden_case(name)
    ref_ids, ref_d, ref_n = data[f"ids_{k}_{nprobe}"], data[f"d_{k}_{nprobe}"], data[f"n_{k}_{nprobe}"]
    cnt = np.isfinite(got["d"]).sum(1).astype(np.uint32)
    assert_topk_equivalent(got["ids"], got["d"], cnt, ref_ids, ref_d, ref_n, 0.0)


class _FakeProbeIndex:
    """Stands in for the GPU index on CPU tensors: probe lists are a fixed function of
    the query row, and the probed search records the probe lists it was handed."""

    def __init__(self, nlist):
        self.nlist = nlist

    @staticmethod
    def _view(ptr, shape, dtype):
        import ctypes as C
        ct = {np.int32: C.c_int32, np.float32: C.c_float, np.int64: C.c_int64}[dtype]
        return np.ctypeslib.as_array(C.cast(ptr, C.POINTER(ct)), shape=shape)

    def probe_device(self, q_ptr, nq, nprobe, probe_ptr, probe_d_ptr):
        q = self._view(q_ptr, (nq, 4), np.float32)
        pr = self._view(probe_ptr, (nq, nprobe), np.int32)
        pd = self._view(probe_d_ptr, (nq, nprobe), np.float32)
        for i in range(nq):
            base = int(q[i, 0])
            pr[i] = [(base * 7 + j) % self.nlist for j in range(nprobe)]
            pd[i] = q[i, 0] + np.arange(nprobe, dtype=np.float32)

    def search_batch_device_probed(self, q_ptr, nq, k, nprobe, probe_ptr, probe_d_ptr, ids_ptr, d_ptr,
                                   counts_ptr=0, mode=0):
        pr = self._view(probe_ptr, (nq, nprobe), np.int32)
        pd = self._view(probe_d_ptr, (nq, nprobe), np.float32)
        ids = self._view(ids_ptr, (nq, k), np.int64)
        d = self._view(d_ptr, (nq, k), np.float32)
        ids[:, :] = pr[:, :k]
        d[:, :] = pd[:, :k]


def _probe_worker(rank, world, port, out_path):
    import sys
    sys.path.insert(0, ROOT)
    import torch
    import torch.distributed as dist

    from vesper_db_b200.shard import probed_search
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        nq, k, nprobe = 12, 3, 5
        q = torch.zeros((nq, 4), dtype=torch.float32)
        q[:, 0] = torch.arange(nq, dtype=torch.float32) * 3
        ids = torch.zeros((nq, k), dtype=torch.int64)
        d = torch.zeros((nq, k), dtype=torch.float32)
        n = torch.zeros(nq, dtype=torch.int32)
        probed_search(_FakeProbeIndex(64), q, k, nprobe, 64, ids, d, n, {})
        np.savez(f"{out_path}.{rank}", ids=ids.numpy(), d=d.numpy())
        dist.barrier()
    finally:
        dist.destroy_process_group()


def _probe_local_worker(rank, world, port, out_path):
    import sys
    sys.path.insert(0, ROOT)
    import torch
    import torch.distributed as dist

    from vesper_db_b200.shard import probed_search
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        nq, k, nprobe = 12, 3, 5
        full = torch.zeros((nq, 4), dtype=torch.float32)
        full[:, 0] = torch.arange(nq, dtype=torch.float32) * 3
        per = nq // world
        local = full[rank * per:(rank + 1) * per].clone()
        q = torch.full((nq, 4), -1.0)       # filled by the gather
        ids = torch.zeros((nq, k), dtype=torch.int64)
        d = torch.zeros((nq, k), dtype=torch.float32)
        n = torch.zeros(nq, dtype=torch.int32)
        times = {}
        probed_search(_FakeProbeIndex(64), q, k, nprobe, 64, ids, d, n, {}, local=local, times=times)
        np.savez(f"{out_path}.{rank}", q=q.numpy(), ids=ids.numpy(), d=d.numpy(),
                 phases=np.array(sorted(times)))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_probed_search_gathers_host_slices(tmp_path):
    """A batch that arrives from the host: each rank holds only its slice (`local`); the
    slices are all-gathered into the full batch with the probe lists, and every rank
    then searches the same full batch."""
    import torch.multiprocessing as mp
    out = str(tmp_path / "probe_local")
    mp.start_processes(_probe_local_worker, args=(2, _free_port(), out), nprocs=2, start_method="spawn")
    full = np.zeros((12, 4), np.float32)
    full[:, 0] = np.arange(12) * 3
    exp_ids = np.array([[(int(i * 3) * 7 + j) % 64 for j in range(3)] for i in range(12)])
    for r in range(2):
        got = np.load(f"{out}.{r}.npz")
        assert np.array_equal(got["q"], full)
        assert np.array_equal(got["ids"], exp_ids)
        assert list(got["phases"]) == ["exchange_ms", "probe_ms", "search_ms"]


def test_probed_search_gathers_every_slice(tmp_path):
    """Two ranks each probe half of the batch; both must search the full batch with the
    probe lists a single rank would have computed."""
    import torch.multiprocessing as mp
    out = str(tmp_path / "probe")
    mp.start_processes(_probe_worker, args=(2, _free_port(), out), nprocs=2, start_method="spawn")
    fake = _FakeProbeIndex(64)
    exp_ids = np.array([[(int(i * 3) * 7 + j) % 64 for j in range(3)] for i in range(12)])
    exp_d = np.array([[i * 3 + j for j in range(3)] for i in range(12)], np.float32)
    for r in range(2):
        got = np.load(f"{out}.{r}.npz")
        assert np.array_equal(got["ids"], exp_ids) and np.array_equal(got["d"], exp_d)
    del fake


def _tau_worker(rank, world, port, out_path):
    import ctypes as C
    import sys
    sys.path.insert(0, ROOT)
    import torch
    import torch.distributed as dist

    from vesper_db_b200.shard import ThresholdExchange
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        inf = np.float32(np.inf)
        vals = [np.array([1.0, inf, 5.0, inf, -2.0], np.float32),
                np.array([3.0, 4.0, 2.0, inf, -1.0], np.float32)][rank]

        def view(ptr, n):
            return torch.from_numpy(np.ctypeslib.as_array(C.cast(ptr, C.POINTER(C.c_float)), (n,)))

        tx = ThresholdExchange(view=view)
        rc = tx(vals.ctypes.data, vals.size, None, None)
        np.savez(f"{out_path}.{rank}", vals=vals, rc=rc, calls=tx.calls)
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_threshold_exchange_takes_the_minimum_over_ranks(tmp_path):
    """The exchange callback leaves the element-wise minimum of every rank's bounds in
    the library's buffer (+inf where no rank has a bound) and reports success."""
    import torch.multiprocessing as mp
    out = str(tmp_path / "tau")
    mp.start_processes(_tau_worker, args=(2, _free_port(), out), nprocs=2, start_method="spawn")
    for r in range(2):
        got = np.load(f"{out}.{r}.npz")
        assert int(got["rc"]) == 0 and int(got["calls"]) == 1
        assert np.array_equal(got["vals"], np.array([1.0, 4.0, 2.0, np.inf, -2.0], np.float32))


@pytest.mark.parametrize("nq,k,world", [(7, 3, 2), (10, 10, 8), (1, 1, 3), (1000, 100, 4)])
def test_shard_results_layout(nq, k, world):
    """The packed per-rank result buffer: the ids view is 8-byte aligned and disjoint
    from the distances and counts, and the (offset, stride) layout handed to the device
    merge finds every part's arrays in the concatenation that an all-gather produces."""
    import torch

    from vesper_db_b200.shard import ShardResults
    rng = np.random.default_rng(nq + k + world)
    parts, want = [], []
    for r in range(world):
        sr = ShardResults(nq, k, "cpu", world=world)
        d = rng.standard_normal((nq, k)).astype(np.float32)
        i = rng.integers(-2**62, 2**62, (nq, k), dtype=np.int64)
        c = rng.integers(0, k + 1, nq).astype(np.int32)
        sr.dist.copy_(torch.from_numpy(d))
        sr.ids.copy_(torch.from_numpy(i))
        sr.counts.copy_(torch.from_numpy(c))
        nk = nq * k
        assert (4 * sr.off_ids) % 8 == 0 and sr.words % 2 == 0          # int64 views stay aligned in every part
        assert 4 * nk <= 4 * sr.off_ids and 4 * sr.off_ids + 8 * nk <= 4 * sr.off_n  # disjoint regions
        assert sr.off_n + nq <= sr.words
        assert np.array_equal(sr.dist.numpy(), d) and np.array_equal(sr.ids.numpy(), i)
        assert np.array_equal(sr.counts.numpy(), c)
        parts.append(sr.buf.numpy().copy())
        want.append((d, i, c))
    g = np.concatenate(parts).tobytes()
    lay = sr.parts_layout()
    for r, (d, i, c) in enumerate(want):
        o, st = lay["dist"]
        got_d = np.frombuffer(g, np.float32, nq * k, o + 4 * r * st).reshape(nq, k)
        o, st = lay["ids"]
        got_i = np.frombuffer(g, np.int64, nq * k, o + 8 * r * st).reshape(nq, k)
        o, st = lay["counts"]
        got_c = np.frombuffer(g, np.int32, nq, o + 4 * r * st)
        assert np.array_equal(got_d, d) and np.array_equal(got_i, i) and np.array_equal(got_c, c)
