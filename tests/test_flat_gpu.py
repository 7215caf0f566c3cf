"""Exact flat top-k (find_nearest_centroids_batch_fused) on the GPU against the oracle.

The GPU path screens every (query, base) pair with tf32 tensor-core products and
re-scores, in the reference's lane order, every column the proven screening bound cannot
rule out, so indices and scores must equal the oracle's bit for bit.  Cases: both
operators; the single-pass path (base <= 16384 rows) and the two-pass path (threshold
from a strided sample, itself searched recursively, then filter + refine); k = 1, 10,
100, 300 and 1024 (the larger kept-column capacity); unit-norm 768-d data shaped like the 1M x 768 inner-product workload;
exact ties (duplicated rows); lists that overflow their capacity (the single-pass
fallback); k > n_base (padding); and the device-pointer entry point.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _flat(op, q, base, k):
    from vesper_db_b200 import flat_topk
    return flat_topk(op, q, base, k)


def _timings():
    from vesper_db_b200.flat import last_timings
    return last_timings()


def _check_equal(op, q, base, k, oracle, single=None):
    gi, gs = _flat(op, q, base, k)
    t = _timings()
    if single is not None:
        assert t["single_pass"] == (1 if single else 0)
    ke = min(k, base.shape[0])
    oi, os_ = oracle.flat_topk(op, q, base, k)
    assert np.array_equal(gi[:, :ke], oi[:, :ke])
    assert np.array_equal(gs[:, :ke], os_[:, :ke])
    return t


@pytest.mark.parametrize("op", [0, 1])
@pytest.mark.parametrize("dim,nb,nq,k", [(128, 5000, 200, 10), (40, 3000, 17, 25), (768, 16000, 64, 100),
                                         (96, 16384, 100, 1)])
def test_single_pass(op, dim, nb, nq, k, oracle):
    rng = np.random.default_rng(dim + nb + op)
    base = rng.standard_normal((nb, dim)).astype(np.float32)
    q = rng.standard_normal((nq, dim)).astype(np.float32)
    _check_equal(op, q, base, k, oracle, single=True)


@pytest.mark.parametrize("op", [0, 1])
@pytest.mark.parametrize("dim,nb,nq,k", [(128, 200000, 300, 100), (64, 150000, 200, 10), (128, 120000, 80, 300),
                                         (96, 65536, 100, 1), (32, 20000, 50, 1024)])
def test_two_pass(op, dim, nb, nq, k, oracle):
    rng = np.random.default_rng(dim + nb + op + k)
    base = rng.standard_normal((nb, dim)).astype(np.float32)
    q = rng.standard_normal((nq, dim)).astype(np.float32)
    t = _check_equal(op, q, base, k, oracle, single=False)
    assert t["overflow_queries"] == 0
    assert t["candidates"] >= nq * k


def test_l2_wide_norm_range(oracle):
    """Two-pass L2 over rows whose norms span four decades, with queries at the origin,
    near it and far out: the augmented screen (||c||^2 folded into the tensor-core
    product) must keep every column the exact top-k needs whatever the norm ratio."""
    rng = np.random.default_rng(77)
    nb, dim, nq, k = 120000, 128, 96, 10
    base = rng.standard_normal((nb, dim)).astype(np.float32)
    base *= (10.0 ** rng.uniform(-2, 2, (nb, 1))).astype(np.float32)
    q = rng.standard_normal((nq, dim)).astype(np.float32)
    q *= (10.0 ** rng.uniform(-3, 2, (nq, 1))).astype(np.float32)
    q[0] = 0.0
    q[1] = base[5]
    t = _check_equal(0, q, base, k, oracle, single=False)
    assert t["overflow_queries"] == 0


def test_unit_norm_inner_product_768(oracle):
    """The 1M x 768 inner-product workload's distribution (N(0,1) rows, L2-normalised)
    at 200k rows."""
    rng = np.random.default_rng(2024)
    base = rng.standard_normal((200000, 768)).astype(np.float32)
    base /= np.linalg.norm(base, axis=1, keepdims=True)
    q = rng.standard_normal((48, 768)).astype(np.float32)
    q /= np.linalg.norm(q, axis=1, keepdims=True)
    t = _check_equal(1, q, base, 100, oracle, single=False)
    assert t["overflow_queries"] == 0


@pytest.mark.parametrize("op", [0, 1])
def test_ties_go_to_the_smaller_index(op, oracle):
    rng = np.random.default_rng(11 + op)
    uniq = rng.standard_normal((30000, 64)).astype(np.float32)
    base = np.concatenate([uniq, uniq[:25000], uniq[:25000]])   # every row of the head three times
    perm = rng.permutation(base.shape[0])
    base = base[perm]
    q = rng.standard_normal((100, 64)).astype(np.float32)
    _check_equal(op, q, base, 50, oracle, single=False)
    _check_equal(op, q, base[:12000], 50, oracle, single=True)


@pytest.mark.parametrize("op", [0, 1])
def test_overflow_uses_single_pass(op, oracle):
    """Four distinct rows repeated 25000 times: every column ties with 24999 others, the
    kept-column lists overflow their 4096 slots, and the single-screen fallback answers."""
    rng = np.random.default_rng(3 + op)
    uniq = rng.standard_normal((4, 32)).astype(np.float32)
    base = np.tile(uniq, (25000, 1))
    q = rng.standard_normal((6, 32)).astype(np.float32)
    t = _check_equal(op, q, base, 20, oracle, single=False)
    assert t["overflow_queries"] == 6


@pytest.mark.parametrize("op", [0, 1])
def test_k_larger_than_base(op, oracle):
    rng = np.random.default_rng(9)
    base = rng.standard_normal((50, 32)).astype(np.float32)
    q = rng.standard_normal((7, 32)).astype(np.float32)
    gi, gs = _flat(op, q, base, 100)
    oi, os_ = oracle.flat_topk(op, q, base, 100)
    assert np.array_equal(gi[:, :50], oi[:, :50]) and np.array_equal(gs[:, :50], os_[:, :50])
    assert np.all(gi[:, 50:] == 0xFFFFFFFF)
    assert np.all(gs[:, 50:] == (np.float32(np.finfo(np.float32).max) * (1 if op == 0 else -1)))


def test_device_entry_point(oracle):
    import torch
    from vesper_db_b200 import flat_topk_device
    rng = np.random.default_rng(21)
    base = rng.standard_normal((100000, 128)).astype(np.float32)
    q = rng.standard_normal((64, 128)).astype(np.float32)
    db, dq = torch.from_numpy(base).cuda(), torch.from_numpy(q).cuda()
    idx = torch.empty((64, 10), dtype=torch.int32, device="cuda")
    sc = torch.empty((64, 10), dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    flat_topk_device(1, dq.data_ptr(), 64, db.data_ptr(), 100000, 128, 10, idx.data_ptr(), sc.data_ptr())
    oi, os_ = oracle.flat_topk(1, q, base, 10)
    assert np.array_equal(idx.cpu().numpy().view(np.uint32), oi)
    assert np.array_equal(sc.cpu().numpy(), os_)


def test_empty_inputs_write_nothing():
    from vesper_db_b200 import flat_topk
    base = np.ones((10, 32), np.float32)
    i, s = flat_topk(0, np.zeros((0, 32), np.float32), base, 5)
    assert i.shape == (0, 5)


@pytest.mark.parametrize("op", [0, 1])
def test_pinned_host_base_equals_device_base(op):
    """With the base in pinned host memory the copy runs in chunks on a second stream
    while the threshold pass and the per-chunk filters run; results must equal the
    device-resident call's bit for bit (two calls, so the reused copy stream and sample
    buffer are exercised)."""
    import ctypes as C

    import torch
    from vesper_db_b200 import _native as N
    from vesper_db_b200 import flat_topk_device
    lib = N.load()
    rng = np.random.default_rng(40 + op)
    for nb, dim, nq, k in [(300000, 128, 96, 100), (120000, 64, 50, 10)]:
        base = torch.from_numpy(rng.standard_normal((nb, dim)).astype(np.float32)).pin_memory()
        q = torch.from_numpy(rng.standard_normal((nq, dim)).astype(np.float32)).pin_memory()
        hi = np.zeros((nq, k), np.uint32)
        hs = np.zeros((nq, k), np.float32)
        f32p = C.POINTER(C.c_float)
        st = lib.vesper_flat_topk(op, C.cast(q.data_ptr(), f32p), nq, C.cast(base.data_ptr(), f32p), nb, dim, k,
                                  hi.ctypes.data_as(C.POINTER(C.c_uint32)), hs.ctypes.data_as(f32p))
        assert st == N.VESPER_OK
        db, dq = base.cuda(), q.cuda()
        di = torch.empty((nq, k), dtype=torch.int32, device="cuda")
        ds = torch.empty((nq, k), dtype=torch.float32, device="cuda")
        torch.cuda.synchronize()
        flat_topk_device(op, dq.data_ptr(), nq, db.data_ptr(), nb, dim, k, di.data_ptr(), ds.data_ptr())
        assert np.array_equal(di.cpu().numpy().view(np.uint32), hi)
        assert np.array_equal(ds.cpu().numpy(), hs)
