"""IndexManager over the GPU IVF-PQ index (vesper_mgr_*, include/vesper_manager.h).

The manager's searches run in EXACT mode (vesper_mgr_set_search_mode) and are compared
with the oracle's restatement of IndexManager::search (Oracle.manager_search) on the
index the manager built, read back from its saved directory: the parameter mapping, the
cand_k rerank heuristic, the tombstone filter and the oversampled re-search must give
the same results, ids equal outside ties at the k-th distance.
"""
import os
import tempfile

import numpy as np
import pytest

from conftest import assert_topk_equivalent

pytestmark = pytest.mark.gpu


def _data(n=20000, d=32, nq=64, seed=3):
    g = np.random.default_rng(seed)
    cent = g.standard_normal((300, d)).astype(np.float32)
    x = (cent[g.integers(0, 300, n)] + 0.25 * g.standard_normal((n, d))).astype(np.float32)
    q = (cent[g.integers(0, 300, nq)] + 0.25 * g.standard_normal((nq, d))).astype(np.float32)
    return x, q


def _model(mgr):
    from oracle_lib import read_ivfpq
    with tempfile.TemporaryDirectory() as td:
        mgr.save(td)
        return read_ivfpq(os.path.join(td, "ivf_pq", "ivfpq.bin"))


def _compare(got_ids, got_d, want, k):
    nq = len(want)
    ref_ids = np.zeros((nq, k), np.uint64)
    ref_d = np.zeros((nq, k), np.float32)
    cnt = np.zeros(nq, np.uint32)
    for i, row in enumerate(want):
        cnt[i] = len(row)
        for j, (vid, dist) in enumerate(row):
            ref_ids[i, j], ref_d[i, j] = vid, dist
    assert_topk_equivalent(got_ids, got_d, cnt, ref_ids, ref_d, cnt, 0.0)
    # padding: id 0 and the last real distance
    for i in range(nq):
        if cnt[i] < k:
            assert np.all(got_ids[i, cnt[i]:] == 0)
            assert np.all(got_d[i, cnt[i]:] == (got_d[i, cnt[i] - 1] if cnt[i] else 0.0))


def _manager(x, **kw):
    from vesper_db_b200 import _native as N
    from vesper_db_b200.manager import IndexManager
    mgr = IndexManager(x.shape[1])
    mgr.build(x, N.INDEX_IVF_PQ, kw.get("strategy", N.SELECT_MANUAL), kw.get("nlist", 64), kw.get("m", 8), 8)
    mgr.set_search_mode(1)
    return mgr


class _Env:
    """Set an environment variable for the duration of a with block."""

    def __init__(self, key, value):
        self.key, self.value = key, value

    def __enter__(self):
        self.old = os.environ.get(self.key)
        if self.value is None:
            os.environ.pop(self.key, None)
        else:
            os.environ[self.key] = self.value

    def __exit__(self, *a):
        if self.old is None:
            os.environ.pop(self.key, None)
        else:
            os.environ[self.key] = self.old


@pytest.mark.parametrize("mode", [None, "id"])
def test_build_search_remove_update(oracle, mode):
    """mode None: the reference's tombstone filter, keyed on the truncated distance of
    each (id, distance) pair (the default, so results equal the reference's); "id"
    (VESPER_MGR_TOMBSTONE_FILTER=id): keyed on the id, removed ids never return."""
    with _Env("VESPER_MGR_TOMBSTONE_FILTER", mode):
        _build_search_remove_update(oracle, mode == "id")


def _build_search_remove_update(oracle, by_id):
    from vesper_db_b200.manager import query_config
    x, q = _data()
    mgr = _manager(x)
    f = _model(mgr)
    args = (f["centroids"], f["rotation"], f["codebooks"], f["m"], f["list_offsets"], f["ids"], f["codes"])
    assert np.array_equal(np.sort(f["ids"]), np.arange(x.shape[0], dtype=np.uint64))   # ids = rows
    for k, npb in [(10, 8), (50, 0), (1, 64)]:
        ids, d = mgr.search_batch(q, query_config(k=k, nprobe=npb))
        _compare(ids, d, oracle.manager_search(q, *args, k, npb), k)
    # removals: tombstoned ids vanish; rows left short are re-searched with k * factor * 1.5
    ids, _ = mgr.search_batch(q, query_config(k=10, nprobe=8))
    dead = np.unique(ids[:, :6].reshape(-1))
    mgr.remove_batch(dead)
    got_ids, got_d = mgr.search_batch(q, query_config(k=10, nprobe=8))
    if by_id:
        assert not np.isin(got_ids[got_ids != 0], dead).any()
    _compare(got_ids, got_d, oracle.manager_search(q, *args, 10, 8, deleted=dead, total_deleted=len(dead),
                                                   filter_by_distance=not by_id), 10)
    # single-query entry point
    i1, d1 = mgr.search(q[3], query_config(k=10, nprobe=8))
    assert np.array_equal(i1[0], got_ids[3]) and np.array_equal(d1[0], got_d[3])
    # update adds another entry under the id (the old one stays)
    target = int(got_ids[0, 0])
    if not by_id:
        return   # the update check below reads ids that the distance-keyed filter may keep
    mgr.update(target, q[0])
    ids2, d2 = mgr.search_batch(q[:1], query_config(k=10, nprobe=8))
    assert ids2[0, 0] == target and d2[0, 0] <= got_d[0, 0]
    st = mgr.get_stats()
    assert len(st) == 1 and st[0]["num_vectors"] == x.shape[0] and st[0]["query_count"] >= 2 * q.shape[0]
    assert mgr.memory_usage() == x.shape[0] * 32 + 256 * x.shape[1] * 4


def test_many_removals_oversample(oracle):
    """Enough tombstones that whole result lists empty out: the oversampling factor
    1 + 1.25 * deleted / 100000 drives the re-searches."""
    from vesper_db_b200.manager import query_config
    x, q = _data(n=30000, seed=8)
    mgr = _manager(x)
    f = _model(mgr)
    args = (f["centroids"], f["rotation"], f["codebooks"], f["m"], f["list_offsets"], f["ids"], f["codes"])
    dead = np.arange(0, 30000, 3, dtype=np.uint64)        # 10000 ids -> factor 1.125
    mgr.remove_batch(dead)
    ids, d = mgr.search_batch(q, query_config(k=20, nprobe=4))
    _compare(ids, d, oracle.manager_search(q, *args, 20, 4, deleted=dead, total_deleted=len(dead)), 20)
    with _Env("VESPER_MGR_TOMBSTONE_FILTER", "id"):
        ids, d = mgr.search_batch(q, query_config(k=20, nprobe=4))
    assert not np.isin(ids[ids != 0], dead).any()
    _compare(ids, d, oracle.manager_search(q, *args, 20, 4, deleted=dead, total_deleted=len(dead),
                                           filter_by_distance=False), 20)


def test_rerank_heuristic_and_env(oracle):
    from vesper_db_b200.manager import query_config
    x, q = _data(seed=5)
    mgr = _manager(x)
    f = _model(mgr)
    args = (f["centroids"], f["rotation"], f["codebooks"], f["m"], f["list_offsets"], f["ids"], f["codes"])
    for k, npb, rk, alpha, ceil_ in [(10, 8, 0, 2.0, 2000), (10, 16, 40, 2.0, 2000), (20, 8, 0, 3.5, 100)]:
        ids, d = mgr.search_batch(q, query_config(k=k, nprobe=npb, use_exact_rerank=True, rerank_k=rk,
                                                  rerank_alpha=alpha, rerank_cand_ceiling=ceil_))
        want = oracle.manager_search(q, *args, k, npb, use_exact_rerank=True, rerank_k=rk, rerank_alpha=alpha,
                                     ceiling=ceil_)
        _compare(ids, d, want, k)
    os.environ["VESPER_USE_EXACT_RERANK"] = "TRUE"
    os.environ["VESPER_RERANK_K"] = "30"
    try:
        ids, d = mgr.search_batch(q, query_config(k=10, nprobe=8))
    finally:
        os.environ.pop("VESPER_USE_EXACT_RERANK", None)
        os.environ.pop("VESPER_RERANK_K", None)
    _compare(ids, d, oracle.manager_search(q, *args, 10, 8, use_exact_rerank=True, rerank_k=30), 10)


def test_save_load_budget_and_refusals(oracle):
    from vesper_db_b200 import VesperError
    from vesper_db_b200 import _native as N
    from vesper_db_b200.manager import IndexManager, query_config
    x, q = _data(seed=9)
    mgr = _manager(x)
    dead = np.array([1, 2, 3, 70000], np.uint64)
    mgr.remove_batch(dead)
    with _Env("VESPER_MGR_TOMBSTONE_FILTER", "id"):
        a = mgr.search_batch(q, query_config(k=10, nprobe=8))
    with tempfile.TemporaryDirectory() as td:
        mgr.save(td)
        assert sorted(os.listdir(td)) == ["index_manager.manifest", "ivf_pq", "tombstones.bin"]
        m2 = IndexManager(7)
        m2.load(td)
        m2.set_search_mode(1)
        # keyed on ids, the reloaded tombstones give the same results
        with _Env("VESPER_MGR_TOMBSTONE_FILTER", "id"):
            b = m2.search_batch(q, query_config(k=10, nprobe=8))
        assert np.array_equal(a[0], b[0]) and np.array_equal(a[1], b[1])
        # the reference's filter after a load: the tombstones are back but the deletion
        # count restarts at zero (a loaded TombstoneManager's statistics start at zero),
        # so no oversampled re-search runs
        f = _model(m2)
        args = (f["centroids"], f["rotation"], f["codebooks"], f["m"], f["list_offsets"], f["ids"], f["codes"])
        got_ids, got_d = m2.search_batch(q, query_config(k=10, nprobe=8))
        _compare(got_ids, got_d, oracle.manager_search(q, *args, 10, 8, deleted=dead, total_deleted=0), 10)
        with pytest.raises(VesperError, match="already marked"):
            m2.remove(2)
    # preferring an index this engine does not hold gives empty (padded) results
    ids, d = mgr.search_batch(q[:2], query_config(k=5, preferred_index=N.INDEX_HNSW))
    assert np.all(ids == 0) and np.all(d == 0)
    with pytest.raises(VesperError, match="not available"):
        mgr.search_batch(q[:2], query_config(k=5, filter_json='{"a": 1}'))
    with pytest.raises(VesperError, match="not available"):
        IndexManager(32).build(x, N.INDEX_HNSW, N.SELECT_MANUAL)
    # the budget compares whole MB of the estimate (n * 32 + 256 * dim * 4 bytes): 0.64 MB
    # fits a budget of 0, 1.3 MB does not and evicts the index
    mgr.set_memory_budget_mb(0)
    assert mgr.get_memory_budget_mb() == 0 and mgr.memory_usage() == 20000 * 32 + 256 * 32 * 4
    big = _manager(_data(n=40000, seed=2)[0])
    big.set_memory_budget_mb(1)
    assert big.memory_usage() > 0
    big.set_memory_budget_mb(0)
    assert big.memory_usage() == 0 and big.get_stats() == []
    with pytest.raises(VesperError, match="No suitable index"):
        big.search_batch(q[:2], query_config(k=5))


def test_auto_build_defaults():
    """AUTO: nlist 512 for n < 100 000, m = 16 when dim % 16 == 0, at most 20 k-means
    iterations; the model the manager saves says so."""
    from vesper_db_b200 import _native as N
    from vesper_db_b200.manager import query_config
    x, q = _data(n=12000, seed=4)
    mgr = _manager(x, strategy=N.SELECT_AUTO, nlist=0, m=0)
    f = _model(mgr)
    assert f["nlist"] == 512 and f["m"] == 16
    ids, d = mgr.search_batch(q, query_config(k=10))
    assert (ids[:, 0] < 12000).all()
