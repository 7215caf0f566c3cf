"""Exact rerank (IvfPqSearchParams::use_exact_rerank / rerank_k / cand_k) on the GPU.

The rerank re-scores the head of the ADC candidate pool with the reference's
reconstruction (centroid + apply_rotation_T(decode(code))) and sequential squared
distance, then re-sorts it (src/index/ivf_pq.cpp:3995-4091).  In EXACT mode the pool is
the reference's, so distances must match bit for bit and ids everywhere except inside a
group of exactly equal distances cut by k (the reference re-sorts with std::sort, whose
order among ties is unspecified).  In FAST mode the pool boundary can differ from the
reference's by ADC ties within fp32 rounding; the reranked distances are still exact.
"""
import os

import numpy as np
import pytest

from conftest import CASES, GOLDEN, assert_topk_equivalent, golden_case

pytestmark = pytest.mark.gpu

RERANK_SEARCHES = [(10, 8, 0, 0), (5, 16, 0, 20), (10, 4, 50, 30), (3, 64, 0, 2), (20, 8, 100, 0)]


def _index():
    from vesper_db_b200 import IvfPqIndex
    return IvfPqIndex()


@pytest.mark.parametrize("name", CASES)
def test_exact_rerank_matches_reference(name):
    from vesper_db_b200 import SEARCH_EXACT
    _, _, data = golden_case(name)
    rr = np.load(os.path.join(GOLDEN, f"ivfpq_{name}_rerank.npz"))
    idx = _index()
    idx.load(os.path.join(GOLDEN, f"ivfpq_{name}"))
    for k, npb, ck, rk in RERANK_SEARCHES:
        tag = f"{k}_{npb}_{ck}_{rk}"
        ids, d, cnt = idx.search_batch(data["queries"], k, npb, mode=SEARCH_EXACT, cand_k=ck,
                                       use_exact_rerank=True, rerank_k=rk)
        assert idx.last_timings()["rerank_ms"] > 0
        assert np.array_equal(cnt, rr[f"n_{tag}"])
        assert_topk_equivalent(ids, d, cnt, rr[f"ids_{tag}"], rr[f"d_{tag}"], rr[f"n_{tag}"], 0.0)


@pytest.mark.parametrize("rot", [False, True])
def test_rerank_vs_oracle_larger(oracle, rot):
    """A larger random model, with and without a rotation, both search modes."""
    from vesper_db_b200 import SEARCH_EXACT
    rng = np.random.default_rng(31 + rot)
    dim, nlist, m, n = 128, 64, 16, 30000
    cent = rng.standard_normal((nlist, dim)).astype(np.float32)
    cb = (0.3 * rng.standard_normal((m * 256, dim // m))).astype(np.float32)
    R = np.linalg.qr(rng.standard_normal((dim, dim)))[0].astype(np.float32) if rot else None
    base = (cent[rng.integers(0, nlist, n)] + 0.3 * rng.standard_normal((n, dim))).astype(np.float32)
    q = (cent[rng.integers(0, nlist, 40)] + 0.3 * rng.standard_normal((40, dim))).astype(np.float32)
    idx = _index()
    idx.set_model(cent, cb, R)
    idx.add(np.arange(n, dtype=np.uint64) * 5 + 11, base)
    offs, lid, codes = idx.lists()
    for k, npb, ck, rk in [(10, 8, 0, 0), (100, 4, 300, 150), (50, 16, 0, 20)]:
        rids, rd, rcnt = oracle.ivfpq_search(q, cent, R, cb, m, offs, lid, codes, k, npb, cand_k=ck, rerank=True,
                                             rerank_k=rk)
        ids, d, cnt = idx.search_batch(q, k, npb, mode=SEARCH_EXACT, cand_k=ck, use_exact_rerank=True, rerank_k=rk)
        assert_topk_equivalent(ids, d, cnt, rids, rd, rcnt, 0.0)
        fids, fd, fcnt = idx.search_batch(q, k, npb, cand_k=ck, use_exact_rerank=True, rerank_k=rk)
        assert np.array_equal(fcnt, rcnt)
        # reranked distances are exact whatever the pool: where the ids agree, so do they
        agree = fids == rids
        if rk == 0 or rk >= k:
            assert agree.mean() > 0.98
            assert np.array_equal(fd[agree], rd[agree])


def test_duplicate_ids_use_the_first_entry(oracle):
    """The reference looks an id up in list order and reuses the first entry it finds
    for every result carrying that id."""
    from vesper_db_b200 import SEARCH_EXACT
    rng = np.random.default_rng(8)
    dim, nlist, m, n = 32, 8, 4, 3000
    cent = rng.standard_normal((nlist, dim)).astype(np.float32)
    cb = (0.3 * rng.standard_normal((m * 256, dim // m))).astype(np.float32)
    base = (cent[rng.integers(0, nlist, n)] + 0.3 * rng.standard_normal((n, dim))).astype(np.float32)
    ids_in = (np.arange(n, dtype=np.uint64) % 700)  # every id four or five times
    q = (cent[rng.integers(0, nlist, 20)] + 0.3 * rng.standard_normal((20, dim))).astype(np.float32)
    idx = _index()
    idx.set_model(cent, cb, None)
    idx.add(ids_in, base)
    offs, lid, codes = idx.lists()
    for k, npb in [(10, 3), (40, 8)]:
        rids, rd, rcnt = oracle.ivfpq_search(q, cent, None, cb, m, offs, lid, codes, k, npb, rerank=True)
        ids, d, cnt = idx.search_batch(q, k, npb, mode=SEARCH_EXACT, use_exact_rerank=True)
        assert_topk_equivalent(ids, d, cnt, rids, rd, rcnt, 0.0)


def test_env_switch_and_limits():
    """VESPER_IVFPQ_RERANK=1 turns the rerank on as in the reference; a pool above 1024
    is refused with a message."""
    from vesper_db_b200 import SEARCH_EXACT, VesperError
    _, _, data = golden_case(CASES[0])
    rr = np.load(os.path.join(GOLDEN, f"ivfpq_{CASES[0]}_rerank.npz"))
    idx = _index()
    idx.load(os.path.join(GOLDEN, f"ivfpq_{CASES[0]}"))
    os.environ["VESPER_IVFPQ_RERANK"] = "1"
    try:
        ids, d, cnt = idx.search_batch(data["queries"], 10, 8, mode=SEARCH_EXACT)
    finally:
        os.environ.pop("VESPER_IVFPQ_RERANK", None)
    assert_topk_equivalent(ids, d, cnt, rr["ids_10_8_0_0"], rr["d_10_8_0_0"], rr["n_10_8_0_0"], 0.0)
    with pytest.raises(VesperError, match="exceeds 1024"):
        idx.search_batch(data["queries"], 400, 8, use_exact_rerank=True)
