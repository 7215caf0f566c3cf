"""The allocation-free search entry point (vesper_ivfpq_search_batch_device_noalloc).

It exists for callers that cannot let the library call cudaMalloc/cudaFree (their own
arena or a framework allocator owns the GPU's memory, or a latency-critical loop must
not synchronize the device).  Its temporaries live in a fixed 64 MiB device array, so
its results must equal those of the ordinary device search, call after call.  This
file is named to be collected last; each test builds its own index, so it passes in
a fresh process as well as after the other tests.
"""
import numpy as np
import pytest

from conftest import assert_topk_equivalent

pytestmark = pytest.mark.gpu

RTOL = 1e-4


def _build(rng, dim=64, nlist=2048, m=32, n=20000, opq=True):
    from vesper_db_b200 import IvfPqIndex
    cent = rng.standard_normal((nlist, dim)).astype(np.float32)
    cb = (0.3 * rng.standard_normal((m * 256, dim // m))).astype(np.float32)
    R = np.linalg.qr(rng.standard_normal((dim, dim)))[0].astype(np.float32) if opq else None
    base = (cent[rng.integers(0, nlist, n)] + 0.3 * rng.standard_normal((n, dim))).astype(np.float32)
    idx = IvfPqIndex()
    idx.set_model(cent, cb, R)
    idx.add(np.arange(n, dtype=np.uint64) * 5 + 1, base)
    q = (cent[rng.integers(0, nlist, 1500)] + 0.3 * rng.standard_normal((1500, dim))).astype(np.float32)
    return idx, q


def _run(fn, q_dev, k, nprobe):
    import torch
    nq = q_dev.shape[0]
    ids = torch.zeros((nq, k), dtype=torch.int64, device=q_dev.device)
    d = torch.zeros((nq, k), dtype=torch.float32, device=q_dev.device)
    n = torch.zeros(nq, dtype=torch.int32, device=q_dev.device)
    fn(q_dev.data_ptr(), nq, k, nprobe, ids.data_ptr(), d.data_ptr(), n.data_ptr())
    torch.cuda.synchronize()
    return ids.cpu().numpy().view(np.uint64), d.cpu().numpy(), n.cpu().numpy().astype(np.uint32)


@pytest.mark.parametrize("opq", [True, False])
def test_noalloc_matches_device_search_twice(opq):
    import torch
    rng = np.random.default_rng(11 if opq else 12)
    # nlist 2048, m 32 -> ~41 KB of scratch per query: 1500 queries need several chunks.
    idx, q = _build(rng, opq=opq)
    q_dev = torch.from_numpy(q).cuda()
    for k, nprobe in [(10, 16), (100, 40)]:
        ref = _run(idx.search_batch_device, q_dev, k, nprobe)
        for _ in range(2):  # two calls in a row share (and reuse) the fixed array
            got = _run(idx.search_batch_device_noalloc, q_dev, k, nprobe)
            assert np.array_equal(got[2], ref[2])
            assert_topk_equivalent(got[0], got[1], got[2], ref[0], ref[1], ref[2], RTOL)


def test_noalloc_rejects_what_does_not_fit():
    import torch
    from vesper_db_b200 import IvfPqIndex, VesperError
    # 17M one-dimensional centroids: one query's distance row alone is 68 MB, more than
    # the 64 MiB array, so the call must fail with a clear error instead of allocating.
    nlist, dim = 17_000_000, 1
    idx = IvfPqIndex()
    idx.set_model(np.zeros((nlist, dim), np.float32), np.zeros((256, 1), np.float32), None)
    q = torch.zeros((4, dim), dtype=torch.float32, device="cuda")
    with pytest.raises(VesperError, match="scratch"):
        _run(idx.search_batch_device_noalloc, q, 5, 4)
