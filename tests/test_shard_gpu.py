"""Sharded search pieces on one GPU, through the C ABI.

* vesper_topk_merge_device against a stable sort of the concatenated parts (the merge
  rule of vesper_db_b200.shard.merge_topk), with ties across parts and short parts.
* The threshold exchange (vesper_ivfpq_set_threshold_exchange): two indexes, each
  holding half of a base set, search the same batch; each one's exchange replaces its
  per-query bounds with the minimum over both (captured from a first pass, since both
  shards live in one process here).  The merged results must equal one index over the
  whole base -- distances to a few ulps (the summation order of an entry's table
  entries follows its position in its list), ids up to ties -- and each shard must
  refine fewer candidates than without the exchange.
"""
import os

import numpy as np
import pytest

from conftest import assert_topk_equivalent

pytestmark = pytest.mark.gpu

# A FAST distance adds the m table entries in an order that depends on the entry's lane
# in its 128-entry block, i.e. on its position in the list, which differs between a shard
# and the whole index: the same entry's distance can differ by a few ulps.
SHARD_RTOL = 1e-5


def _merge_device(d, ids, cnt, k):
    """d/ids [parts, nq, k] and cnt [parts, nq] (torch CUDA) -> merged (d, ids, cnt)."""
    import torch

    from vesper_db_b200 import _native as N
    from vesper_db_b200.index import _check
    parts, nq, _ = d.shape
    out_i = torch.empty((nq, k), dtype=torch.int64, device=d.device)
    out_d = torch.empty((nq, k), dtype=torch.float32, device=d.device)
    out_n = torch.empty(nq, dtype=torch.int32, device=d.device)
    lib = N.load()
    _check(lib, lib.vesper_topk_merge_device(parts, nq, k, d.data_ptr(), nq * k, ids.data_ptr(), nq * k,
                                             cnt.data_ptr(), nq, out_i.data_ptr(), out_d.data_ptr(),
                                             out_n.data_ptr(), torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    return out_d.cpu().numpy(), out_i.cpu().numpy(), out_n.cpu().numpy()


@pytest.mark.parametrize("parts,nq,k", [(1, 50, 10), (2, 300, 10), (8, 1000, 100), (3, 7, 1)])
def test_topk_merge_matches_stable_sort(parts, nq, k):
    import torch
    rng = np.random.default_rng(parts * 1000 + k)
    # few distinct values: many ties within and across parts
    d = np.sort(rng.integers(0, 20, (parts, nq, k)).astype(np.float32), axis=2)
    ids = rng.integers(0, 1 << 40, (parts, nq, k)).astype(np.int64)
    cnt = rng.integers(0, k + 1, (parts, nq)).astype(np.int32)
    cnt[0, 0] = k
    got_d, got_i, got_n = _merge_device(torch.from_numpy(d).cuda(), torch.from_numpy(ids).cuda(),
                                        torch.from_numpy(cnt).cuda(), k)
    for q in range(nq):
        cd = np.concatenate([d[p, q, :cnt[p, q]] for p in range(parts)])
        ci = np.concatenate([ids[p, q, :cnt[p, q]] for p in range(parts)])
        order = np.argsort(cd, kind="stable")[:k]
        n = len(order)
        assert got_n[q] == n
        assert np.array_equal(got_d[q, :n], cd[order]) and np.array_equal(got_i[q, :n], ci[order])
        # padding like vesper_ivfpq_search_batch: id 0, the last real distance (0 if none)
        assert np.all(got_i[q, n:] == 0)
        assert np.all(got_d[q, n:] == (cd[order][-1] if n else 0.0))


class _DevView:
    def __init__(self, ptr, n):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": "<f4", "data": (ptr, False), "version": 2}


def _hook(store, other=None):
    """A threshold exchange for shards in one process: record this shard's bounds, or
    replace them with the minimum against the other shard's recorded bounds."""
    import torch

    def fn(ptr, n, stream, user):
        t = torch.as_tensor(_DevView(ptr, n), device="cuda")
        with torch.cuda.stream(torch.cuda.ExternalStream(stream)):
            if other is None:
                store.append(t.clone())
            else:
                torch.minimum(t, other[-1], out=t)
                store.append(None)
        return 0
    return fn


def _with_env(key, val, f):
    old = os.environ.get(key)
    os.environ[key] = val
    try:
        return f()
    finally:
        if old is None:
            os.environ.pop(key, None)
        else:
            os.environ[key] = old


@pytest.mark.parametrize("split", [False, True])
@pytest.mark.parametrize("dim,m,nlist,n,nq,rot,k,npb", [
    (128, 16, 64, 40000, 300, True, 10, 8),
    (128, 32, 48, 60000, 256, False, 100, 12),
])
def test_threshold_exchange_keeps_the_union_top_k(dim, m, nlist, n, nq, rot, k, npb, split):
    """split: each shard runs its own threshold pass only for its half of the queries
    (q % 2 == shard) and takes the other half's bounds from the exchange."""
    import torch

    from vesper_db_b200 import IvfPqIndex
    rng = np.random.default_rng(dim + m + nlist)
    cent = rng.standard_normal((nlist, dim)).astype(np.float32)
    cb = (0.3 * rng.standard_normal((m * 256, dim // m))).astype(np.float32)
    R = np.linalg.qr(rng.standard_normal((dim, dim)))[0].astype(np.float32) if rot else None
    base = (cent[rng.integers(0, nlist, n)] + 0.3 * rng.standard_normal((n, dim))).astype(np.float32)
    ids = np.arange(n, dtype=np.uint64) * 7 + 3
    q = (cent[rng.integers(0, nlist, nq)] + 0.3 * rng.standard_normal((nq, dim))).astype(np.float32)
    chunk = 1000
    part = (np.arange(n) // chunk) % 2
    shards, whole = [], IvfPqIndex()
    whole.set_model(cent, cb, R)
    whole.add(ids, base)
    for r in range(2):
        ix = IvfPqIndex()
        ix.set_model(cent, cb, R)
        ix.add(ids[part == r], base[part == r])
        shards.append(ix)

    def search(ix):
        out = ix.search_batch(q, k, npb)
        t = ix.last_timings()
        assert t["scan_variant"] == 4
        return out, t["list_candidates"]

    def run():
        ref, _ = search(whole)
        plain = [search(ix) for ix in shards]
        taus = [[], []]
        part_args = (lambda r: (r, 2)) if split else (lambda r: (0, 1))
        for r in range(2):                       # pass 1: record each shard's bounds
            shards[r].set_threshold_exchange(_hook(taus[r]), *part_args(r))
            search(shards[r])
        calls = [[], []]
        for r in range(2):                       # pass 2: the minimum over both shards
            shards[r].set_threshold_exchange(_hook(calls[r], taus[1 - r]), *part_args(r))
        shared = [search(ix) for ix in shards]
        for ix in shards:
            ix.set_threshold_exchange(None)
        return ref, plain, shared, taus, calls

    ref, plain, shared, taus, calls = _with_env("VGPU_SCAN", "tc", run)
    assert all(len(c) == 1 for c in calls) and all(len(t) == 1 for t in taus)
    tau_min = torch.minimum(taus[0][0], taus[1][0])
    assert torch.isfinite(tau_min).all()
    if split:   # each shard bounded only its own half (every nearest list here holds >= 4k entries per shard)
        for r in range(2):
            own = torch.arange(nq, device=taus[r][0].device) % 2 == r
            assert torch.isinf(taus[r][0][~own]).all() and torch.isfinite(taus[r][0][own]).all()
    for variant in (plain, shared):
        d = torch.from_numpy(np.stack([variant[r][0][1] for r in range(2)])).cuda()
        i = torch.from_numpy(np.stack([variant[r][0][0].astype(np.int64) for r in range(2)])).cuda()
        c = torch.from_numpy(np.stack([variant[r][0][2].astype(np.int32) for r in range(2)])).cuda()
        md, mi, mn = _merge_device(d, i, c, k)
        assert_topk_equivalent(mi.astype(np.uint64), md, mn, ref[0], ref[1], ref[2], SHARD_RTOL)
    if not split:   # each shard's bound is at least as tight as its own
        assert sum(s[1] for s in shared) < sum(p[1] for p in plain)


def test_exchange_sees_no_bound_without_the_list_scan():
    """A search that does not run the list scan still calls the exchange once per chunk,
    with +inf for every query, so the shards' calls pair up."""
    from vesper_db_b200 import IvfPqIndex
    rng = np.random.default_rng(5)
    dim, m, nlist, n, nq = 64, 8, 16, 5000, 40
    cent = rng.standard_normal((nlist, dim)).astype(np.float32)
    cb = (0.3 * rng.standard_normal((m * 256, dim // m))).astype(np.float32)
    base = (cent[rng.integers(0, nlist, n)] + 0.3 * rng.standard_normal((n, dim))).astype(np.float32)
    ix = IvfPqIndex()
    ix.set_model(cent, cb, None)
    ix.add(np.arange(n, dtype=np.uint64), base)
    seen = []
    ix.set_threshold_exchange(_hook(seen))
    a = _with_env("VGPU_SCAN", "blocked", lambda: ix.search_batch(base[:nq], 10, 4))
    ix.set_threshold_exchange(None)
    b = _with_env("VGPU_SCAN", "blocked", lambda: ix.search_batch(base[:nq], 10, 4))
    assert len(seen) == 1 and bool((seen[0] == float("inf")).all())
    assert all(np.array_equal(x, y) for x, y in zip(a, b))


def test_failed_exchange_fails_the_search():
    from vesper_db_b200 import IvfPqIndex
    rng = np.random.default_rng(6)
    dim, m, nlist, n = 64, 8, 16, 5000
    cent = rng.standard_normal((nlist, dim)).astype(np.float32)
    cb = (0.3 * rng.standard_normal((m * 256, dim // m))).astype(np.float32)
    base = (cent[rng.integers(0, nlist, n)] + 0.3 * rng.standard_normal((n, dim))).astype(np.float32)
    ix = IvfPqIndex()
    ix.set_model(cent, cb, None)
    ix.add(np.arange(n, dtype=np.uint64), base)
    ix.set_threshold_exchange(lambda ptr, nq, stream, user: 1)
    with pytest.raises(Exception, match="threshold exchange"):
        ix.search_batch(base[:10], 5, 4)
    ix.set_threshold_exchange(None)
    ix.search_batch(base[:10], 5, 4)
