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


SCRATCH_BYTES = 64 << 20   # the library's fixed array
NQ = 3500


def _queries_per_chunk(dim, nlist, m, nprobe, opq):
    """Queries one pass over the fixed array holds (the entry point's own carving:
    distance row, probe ids and distances, rotated query, lookup table per query, and
    1 KiB of alignment slack)."""
    per_q = nlist * 4 + nprobe * 8 + (dim * 4 if opq else 0) + m * 256 * 4
    return (SCRATCH_BYTES - 1024) // per_q


def _build(rng, dim=64, nlist=2048, m=32, n=20000, opq=True, nq=NQ):
    from vesper_db_b200 import IvfPqIndex
    cent = rng.standard_normal((nlist, dim)).astype(np.float32)
    cb = (0.3 * rng.standard_normal((m * 256, dim // m))).astype(np.float32)
    R = np.linalg.qr(rng.standard_normal((dim, dim)))[0].astype(np.float32) if opq else None
    base = (cent[rng.integers(0, nlist, n)] + 0.3 * rng.standard_normal((n, dim))).astype(np.float32)
    idx = IvfPqIndex()
    idx.set_model(cent, cb, R)
    idx.add(np.arange(n, dtype=np.uint64) * 5 + 1, base)
    q = (cent[rng.integers(0, nlist, nq)] + 0.3 * rng.standard_normal((nq, dim))).astype(np.float32)
    return idx, q, (cent, cb, R, m)


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
    # nlist 2048, m 32 -> ~41 KB of scratch per query: 3500 queries take three passes,
    # so the later passes' query, output and count offsets are exercised.
    idx, q, _ = _build(rng, opq=opq)
    q_dev = torch.from_numpy(q).cuda()
    for k, nprobe in [(10, 16), (100, 40)]:
        assert NQ > 2 * _queries_per_chunk(64, 2048, 32, nprobe, opq)
        ref = _run(idx.search_batch_device, q_dev, k, nprobe)
        for _ in range(2):  # two calls in a row share (and reuse) the fixed array
            got = _run(idx.search_batch_device_noalloc, q_dev, k, nprobe)
            assert np.array_equal(got[2], ref[2])
            assert_topk_equivalent(got[0], got[1], got[2], ref[0], ref[1], ref[2], RTOL)


def test_noalloc_matches_oracle(oracle):
    """Pinned to the oracle as well: the allocation-free results equal the reference's
    arithmetic within the FAST tolerance, across several passes over the array."""
    import torch
    rng = np.random.default_rng(13)
    idx, q, (cent, cb, R, m) = _build(rng, opq=True)
    offs, lid, codes = idx.lists()
    q_dev = torch.from_numpy(q).cuda()
    k, nprobe = 20, 24
    assert NQ > 2 * _queries_per_chunk(64, 2048, 32, nprobe, True)
    rids, rd, rcnt = oracle.ivfpq_search(q, cent, R, cb, m, offs, lid, codes, k, nprobe)
    for _ in range(2):
        ids, d, n = _run(idx.search_batch_device_noalloc, q_dev, k, nprobe)
        assert_topk_equivalent(ids, d, n, rids, rd, rcnt, RTOL)


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


def test_noalloc_rejects_table_beyond_shared_memory():
    """m = 256 sub-quantizers x 2^8 codes: the 256 KiB per-query lookup table fits the
    array but not the scan kernel's shared memory, so the call is refused before it
    queues any work -- and the next call on the same array still gives right results."""
    import torch
    from vesper_db_b200 import IvfPqIndex, VesperError
    rng = np.random.default_rng(14)
    dim = m = 256
    big = IvfPqIndex()
    big.set_model(rng.standard_normal((64, dim)).astype(np.float32),
                  rng.standard_normal((m * 256, 1)).astype(np.float32), None)
    q = torch.zeros((8, dim), dtype=torch.float32, device="cuda")
    with pytest.raises(VesperError, match="shared memory"):
        _run(big.search_batch_device_noalloc, q, 10, 4)
    idx, qq, _ = _build(rng, opq=False, nq=300)
    q_dev = torch.from_numpy(qq).cuda()
    ref = _run(idx.search_batch_device, q_dev, 10, 8)
    got = _run(idx.search_batch_device_noalloc, q_dev, 10, 8)
    assert_topk_equivalent(got[0], got[1], got[2], ref[0], ref[1], ref[2], RTOL)
