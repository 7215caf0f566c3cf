"""GPU k-means (vesper_kmeans_fit / _fit_device) against the reference.

Assignments, iteration counts and centroids must equal the reference's bit for bit:
k-means++ draws the same rows (host std::mt19937, device D^2 in reference lane order),
the E-step is exact (tensor-core screen + exact refine, or the CUDA-core kernel), and
the M-step sums in point order in fp64.  Elkan's returned inertia is the reference's
(fp64 sum cast to float); Lloyd's final inertia is an fp64 sum where the reference
keeps a float running total, so it is compared within that total's rounding.
"""
import os

import numpy as np
import pytest

from conftest import GOLDEN

pytestmark = pytest.mark.gpu

INERTIA_RTOL = 1e-5  # Lloyd final inertia vs an fp64 evaluation of the same clustering


def _inertia64(x, c, a):
    d = x.astype(np.float64) - c.astype(np.float64)[a]
    return float((d * d).sum())


def _check_lloyd_inertia(got, x, c, a, ref_inertia):
    """The engine's inertia is an fp64 sum; the reference's is a float running sum over
    n * dim terms, whose rounding is bounded by n * dim * 2^-24 relative."""
    exact = _inertia64(x, c, a)
    assert abs(got - exact) <= INERTIA_RTOL * exact
    assert abs(ref_inertia - exact) <= x.size * 2.0 ** -24 * exact


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
    _check_lloyd_inertia(lo.inertia, x, g["lloyd_c"], g["lloyd_a"], float(g["lloyd_inertia"]))


@pytest.mark.parametrize("n,d,k,iters", [(20000, 64, 256, 6), (12000, 128, 512, 4), (5000, 20, 100, 5)])
def test_lloyd_matches_oracle(oracle, n, d, k, iters):
    """k >= 64 with d % 4 == 0 runs the tcgen05 screen; d = 20 the CUDA-core kernel."""
    from vesper_db_b200 import kmeans_cluster
    x = _mixture(n, d, 3 * k, 0.05, 31 + d)
    c, a, it, inertia = oracle.kmeans_lloyd(x, k, iters, 0.0, 42)
    got = kmeans_cluster(x, k, iters, 0.0, 42)
    assert np.array_equal(got.assignments, a)
    assert np.array_equal(got.centroids, c)
    assert got.iterations == it
    _check_lloyd_inertia(got.inertia, x, c, a, inertia)


def test_elkan_matches_oracle_tensor_core_path(oracle):
    from vesper_db_b200 import kmeans_elkan
    x = _mixture(16000, 96, 600, 0.08, 5)
    c, a, it, inertia = oracle.kmeans_elkan(x, 300, 25, 1e-4, 42)
    got = kmeans_elkan(x, 300, 25, 1e-4, 42)
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
