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
