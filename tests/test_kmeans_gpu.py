"""GPU k-means (vesper_kmeans_fit / _fit_device) against the reference.

Assignments, iteration counts and centroids must equal the reference's bit for bit:
k-means++ draws the same rows (host std::mt19937, device D^2 in reference lane order),
the E-step is exact (tensor-core screen + exact refine, or the CUDA-core kernel), and
the M-step sums in point order in fp64.  Elkan's returned inertia is the reference's
(fp64 sum cast to float); Lloyd's final inertia is the reference's float running total
over every (point, dimension) term, so both inertias are compared exactly.
The sharded fit (vesper_db_b200.shard.kmeans_fit_sharded) must equal the one-GPU fit,
with several shards in one process and, where two GPUs are visible, over NCCL.
"""
import os
import socket

import numpy as np
import pytest

from conftest import GOLDEN, ROOT

pytestmark = pytest.mark.gpu


def _check_lloyd_inertia(got, ref_inertia):
    assert np.float32(got) == np.float32(ref_inertia)


def _mixture(n, d, ncent, sigma, seed):
    g = np.random.default_rng(seed)
    cent = g.uniform(-1, 1, (ncent, d)).astype(np.float32)
    lab = g.integers(0, ncent, n)
    return (cent[lab] + sigma * g.standard_normal((n, d))).astype(np.float32)


def test_golden_elkan_and_lloyd():
    from vesper_db_b200 import kmeans_cluster, kmeans_elkan
    g = dict(np.load(os.path.join(GOLDEN, "kmeans_small.npz")))
    x = g["x"]
    e = kmeans_elkan(x, 48, 25, 1e-4, 42)
    assert np.array_equal(e.assignments, g["elkan_a"])
    assert np.array_equal(e.centroids, g["elkan_c"])
    assert e.iterations == int(g["elkan_it"]) and np.float32(e.inertia) == np.float32(g["elkan_inertia"])
    assert np.array_equal(e.cluster_sizes, np.bincount(g["elkan_a"], minlength=48))
    lo = kmeans_cluster(x, 48, 20, 0.0, 42)
    assert np.array_equal(lo.assignments, g["lloyd_a"])
    assert np.array_equal(lo.centroids, g["lloyd_c"])
    assert lo.iterations == int(g["lloyd_it"])
    _check_lloyd_inertia(lo.inertia, float(g["lloyd_inertia"]))


def _with_kpp(mode, fn):
    old = os.environ.get("VGPU_KPP")
    os.environ["VGPU_KPP"] = mode
    try:
        return fn()
    finally:
        if old is None:
            os.environ.pop("VGPU_KPP", None)
        else:
            os.environ["VGPU_KPP"] = old


@pytest.mark.parametrize("n,d,k", [(60000, 64, 600), (30000, 20, 300), (4099, 128, 64)])
def test_kmeanspp_device_draws_equal_host_draws(oracle, n, d, k):
    """k-means++ with the prefix sums and the lower_bound on the device (the path large
    n * k takes) picks the same rows as the host sampler and the oracle, which recompute
    the reference's fp64 prefix sum in point order for every draw."""
    from vesper_db_b200 import kmeans_cluster
    x = _mixture(n, d, 2 * k, 0.05, 7 + d)
    host = _with_kpp("host", lambda: kmeans_cluster(x, k, 2, 0.0, 42))
    dev = _with_kpp("device", lambda: kmeans_cluster(x, k, 2, 0.0, 42))
    c, a, it, inertia = oracle.kmeans_lloyd(x, k, 2, 0.0, 42)
    for got in (host, dev):
        assert np.array_equal(got.centroids, c)
        assert np.array_equal(got.assignments, a)
        assert got.iterations == it
        _check_lloyd_inertia(got.inertia, inertia)


def test_lloyd_zero_iterations_matches_reference(oracle, reference):
    """max_iter = 0: no iteration runs; the final update reads the assignment vector as
    the reference initialises it (all points in cluster 0)."""
    from vesper_db_b200 import kmeans_cluster
    x = _mixture(3000, 32, 60, 0.05, 5)
    c, a, it, inertia = reference.kmeans_lloyd(x, 20, 0, 0.0, 42)
    got = kmeans_cluster(x, 20, 0, 0.0, 42)
    assert it == 0 and got.iterations == 0
    assert np.array_equal(got.assignments, a)
    assert np.array_equal(got.centroids, c)


@pytest.mark.parametrize("n,d,k,iters", [(20000, 64, 256, 6), (12000, 128, 512, 4), (5000, 20, 100, 5),
                                         (30000, 64, 2048, 3), (24000, 32, 4100, 2)])
def test_lloyd_matches_oracle(oracle, n, d, k, iters):
    """k >= 64 with d % 4 == 0 runs the tcgen05 screen (k <= 1024: one screen of every
    centroid; above: the filter against a sampled threshold); d = 20 the CUDA-core kernel."""
    from vesper_db_b200 import kmeans_cluster
    x = _mixture(n, d, 3 * k, 0.05, 31 + d)
    c, a, it, inertia = oracle.kmeans_lloyd(x, k, iters, 0.0, 42)
    got = kmeans_cluster(x, k, iters, 0.0, 42)
    assert np.array_equal(got.assignments, a)
    assert np.array_equal(got.centroids, c)
    assert got.iterations == it
    _check_lloyd_inertia(got.inertia, inertia)


@pytest.mark.parametrize("n,d,k,dup", [(16000, 96, 300, False), (30000, 64, 2000, True)])
def test_elkan_matches_oracle_tensor_core_path(oracle, n, d, k, dup):
    """k = 2000 runs the filter path, with duplicated points so that centroids tie and
    the keep-on-tie rule decides."""
    from vesper_db_b200 import kmeans_elkan
    x = _mixture(n, d, 2 * k, 0.08, 5)
    if dup:
        x[1::5] = x[0::5][: x[1::5].shape[0]]
    c, a, it, inertia = oracle.kmeans_elkan(x, k, 25, 1e-4, 42)
    got = kmeans_elkan(x, k, 25, 1e-4, 42)
    assert np.array_equal(got.assignments, a) and np.array_equal(got.centroids, c)
    assert got.iterations == it and np.float32(got.inertia) == np.float32(inertia)


def test_device_entry_matches_host_entry():
    import torch

    from vesper_db_b200 import kmeans_cluster, kmeans_fit_device
    from vesper_db_b200._native import KMEANS_LLOYD
    x = _mixture(8000, 64, 300, 0.05, 77)
    host = kmeans_cluster(x, 128, 5, 0.0, 9)
    dx = torch.from_numpy(x).cuda()
    dc = torch.empty((128, 64), dtype=torch.float32, device="cuda")
    da = torch.empty(8000, dtype=torch.int32, device="cuda")
    torch.cuda.synchronize()
    it, inertia = kmeans_fit_device(dx.data_ptr(), 8000, 64, 128, dc.data_ptr(), da.data_ptr(), 5, 0.0, 9,
                                    KMEANS_LLOYD)
    assert it == host.iterations and inertia == host.inertia
    assert np.array_equal(dc.cpu().numpy(), host.centroids)
    assert np.array_equal(da.cpu().numpy().view(np.uint32), host.assignments)


def _splits(n, parts):
    cuts = [0] + sorted(np.random.default_rng(n).choice(np.arange(1, n), parts - 1, replace=False).tolist()) + [n]
    return list(zip(cuts[:-1], cuts[1:]))


@pytest.mark.parametrize("algorithm", [0, 1])
@pytest.mark.parametrize("n,d,k,iters,parts", [(16000, 96, 300, 8, 3), (5000, 20, 100, 6, 2)])
def test_sharded_fit_equals_single_gpu(algorithm, n, d, k, iters, parts):
    """Several shards in one process: the chained mean update and the gathered inertia
    reproduce the one-GPU fit (tensor-core E-step at d = 96, CUDA-core at d = 20)."""
    import torch

    from vesper_db_b200 import kmeans_fit_device
    from vesper_db_b200.shard import kmeans_fit_sharded
    x = _mixture(n, d, 3 * k, 0.06, 11 + d)
    dx = torch.from_numpy(x).cuda()
    dc = torch.empty((k, d), dtype=torch.float32, device="cuda")
    da = torch.empty(n, dtype=torch.int32, device="cuda")
    eps = 1e-4 if algorithm == 0 else 0.0
    torch.cuda.synchronize()
    it, inertia = kmeans_fit_device(dx.data_ptr(), n, d, k, dc.data_ptr(), da.data_ptr(), iters, eps, 42, algorithm)
    shards = [dx[a:b] for a, b in _splits(n, parts)]
    c, asg, it2, inertia2 = kmeans_fit_sharded(shards, k, iters, eps, 42, algorithm)
    assert it2 == it and np.float32(inertia2) == np.float32(inertia)
    assert torch.equal(c, dc)
    assert torch.equal(torch.cat(asg), da)


def test_sharded_fit_golden():
    import torch

    from vesper_db_b200.shard import kmeans_fit_sharded
    g = np.load(os.path.join(GOLDEN, "kmeans_small.npz"))
    dx = torch.from_numpy(g["x"]).cuda()
    c, asg, it, inertia = kmeans_fit_sharded([dx[:700], dx[700:2100], dx[2100:]], 48, 25, 1e-4, 42, 0)
    assert np.array_equal(c.cpu().numpy(), g["elkan_c"])
    assert np.array_equal(torch.cat(asg).cpu().numpy().view(np.uint32), g["elkan_a"])
    assert it == int(g["elkan_it"]) and np.float32(inertia) == np.float32(g["elkan_inertia"])


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _nccl_worker(rank, world, port, out_path, algorithm):
    import sys
    from datetime import timedelta
    sys.path.insert(0, ROOT)
    import torch
    import torch.distributed as dist

    from vesper_db_b200.shard import kmeans_fit_sharded
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    try:
        x = _mixture(24000, 64, 600, 0.06, 5)
        per = [(0, 9000), (9000, 24000)]
        a, b = per[rank]
        dx = torch.from_numpy(x[a:b]).cuda()
        eps = 1e-4 if algorithm == 0 else 0.0
        c, asg, it, inertia = kmeans_fit_sharded([dx], 200, 6, eps, 42, algorithm)
        parts = [torch.zeros(15000, dtype=torch.int32, device="cuda") for _ in range(world)]
        mine = torch.zeros(15000, dtype=torch.int32, device="cuda")
        mine[:asg[0].shape[0]] = asg[0]
        dist.all_gather(parts, mine)
        if rank == 0:
            allv = torch.cat([parts[0][:9000], parts[1][:15000]])
            np.savez(out_path, c=c.cpu().numpy(), a=allv.cpu().numpy(), it=it, inertia=inertia)
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(600)
@pytest.mark.parametrize("algorithm", [0, 1])
def test_two_gpu_sharded_fit_equals_single_gpu(tmp_path, algorithm):
    import torch
    import torch.multiprocessing as mp

    from vesper_db_b200 import kmeans_fit_device
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    out = str(tmp_path / "km2.npz")
    mp.start_processes(_nccl_worker, args=(2, _free_port(), out, algorithm), nprocs=2, join=True,
                       start_method="spawn")
    r = np.load(out)
    x = _mixture(24000, 64, 600, 0.06, 5)
    dx = torch.from_numpy(x).cuda()
    dc = torch.empty((200, 64), dtype=torch.float32, device="cuda")
    da = torch.empty(24000, dtype=torch.int32, device="cuda")
    torch.cuda.synchronize()
    eps = 1e-4 if algorithm == 0 else 0.0
    it, inertia = kmeans_fit_device(dx.data_ptr(), 24000, 64, 200, dc.data_ptr(), da.data_ptr(), 6, eps, 42,
                                    algorithm)
    assert int(r["it"]) == it and np.float32(r["inertia"]) == np.float32(inertia)
    assert np.array_equal(r["c"], dc.cpu().numpy())
    assert np.array_equal(r["a"], da.cpu().numpy())


@pytest.mark.parametrize("keep", [False, True])
def test_fused_argmin_ties_and_overflow(oracle, keep):
    """The fused tensor-core arg-min (tc_argmin_kernel) against the oracle's exact
    arg-min: five centroids repeated 20 more times give rows more exact ties than the
    kernel's per-row candidate list holds (those rows take the overflow path), the rest
    are ordinary; with keep_on_tie, a point whose current centroid ties its nearest
    keeps it (KmeansElkan's rule), any other point moves to the lowest index."""
    import torch

    from vesper_db_b200.shard import GpuKmeansOps
    rng = np.random.default_rng(3)
    d, kb, n = 64, 200, 50000
    base_c = rng.uniform(-1, 1, (kb, d)).astype(np.float32)
    c = np.concatenate([base_c, np.repeat(base_c[:5], 20, axis=0)])
    x = (base_c[rng.integers(0, kb, n)] + 0.05 * rng.standard_normal((n, d))).astype(np.float32)
    ref = oracle.assign(x, c)
    dup = ref < 5
    assert dup.sum() > 500
    init = np.where(dup, kb + 20 * ref.astype(np.int64) + 19, (ref.astype(np.int64) + 1) % kb).astype(np.uint32)
    ops = GpuKmeansOps()
    xt, ct = torch.from_numpy(x).cuda(), torch.from_numpy(c).cuda()
    a = torch.from_numpy(init.view(np.int32).copy()).cuda()
    m = torch.empty(n, dtype=torch.float32, device="cuda")
    ops.assign(xt, ct, keep, a, m)
    torch.cuda.synchronize()
    got = a.cpu().numpy().view(np.uint32)
    want = np.where(dup, init, ref) if keep else ref
    assert np.array_equal(got, want)
    dist = np.array([oracle.l2_sq(x[i], c[ref[i]]) for i in range(0, n, 97)], np.float32)
    assert np.array_equal(m.cpu().numpy()[::97], dist)
    ops.close()


def test_fused_argmin_wide_norm_range(oracle):
    """The fused arg-min (augmented screen: ||c||^2 inside the tensor-core product)
    against the oracle when centroid norms span four decades and points sit at, near
    and far from the origin."""
    import torch

    from vesper_db_b200.shard import GpuKmeansOps
    rng = np.random.default_rng(5)
    d, k, n = 96, 700, 40000
    c = rng.standard_normal((k, d)).astype(np.float32)
    c *= (10.0 ** rng.uniform(-2, 2, (k, 1))).astype(np.float32)
    x = c[rng.integers(0, k, n)] + rng.standard_normal((n, d)).astype(np.float32) * \
        (10.0 ** rng.uniform(-3, 1, (n, 1))).astype(np.float32)
    x[:50] *= np.float32(1e-4)
    x[50] = 0.0
    x = x.astype(np.float32)
    ref = oracle.assign(x, c)
    ops = GpuKmeansOps()
    xt, ct = torch.from_numpy(x).cuda(), torch.from_numpy(c).cuda()
    a = torch.zeros(n, dtype=torch.int32, device="cuda")
    m = torch.empty(n, dtype=torch.float32, device="cuda")
    ops.assign(xt, ct, False, a, m)
    torch.cuda.synchronize()
    assert np.array_equal(a.cpu().numpy().view(np.uint32), ref)
    dist = np.array([oracle.l2_sq(x[i], c[ref[i]]) for i in range(0, n, 89)], np.float32)
    assert np.array_equal(m.cpu().numpy()[::89], dist)
    ops.close()
