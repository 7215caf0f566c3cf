"""FAST and EXACT search at the benchmark shapes against the oracle and the reference.

The other parity files pin the arithmetic on small shapes (d <= 64).  This file runs
the two shapes the benchmark workloads use, on a GPU-trained model, through the C ABI:

* d = 768, m = 96 (8-dim sub-vectors), OPQ rotation learnt on the GPU, lists of about
  2,000 entries, 1,024 queries from an anisotropic mixture -- the IVF-PQ+OPQ search
  workload at reduced N.  FAST search runs through the tensor-core list scan
  (VGPU_SCAN=tc) and through the blocked scan (VGPU_SCAN=blocked);
* d = 128, m = 32 (4-dim sub-vectors: the reference's AVX2 l2 has no 8-lane body and
  is all scalar tail, src/kernels/backends/avx2.hpp:76-108), k = 100 (the reference's
  heap branch for a pool above 64, src/index/ivf_pq.cpp:3539,3821-3829) -- the sharded
  100M-vector workload's shape at reduced N.

Bars (the engine's contract with the reference's IvfPqIndex::search,
src/index/ivf_pq.cpp:3491-4094): EXACT distances bit-exact and ids equal outside exact
ties; FAST distances within 1e-4 relative (floor 1) and id sets equal outside ties
within that band; the list scan bit-identical to the blocked scan.  Where the reference
library is built (oracle/_ref) the same model is loaded into the reference's own
IvfPqIndex through its v1.0 file and searched there as well.
"""
import os
import tempfile

import numpy as np
import pytest

from conftest import assert_topk_equivalent

pytestmark = pytest.mark.gpu

RTOL = 1e-4


def _mixture(rng, n_centres, dim, n, nq):
    centres = rng.uniform(-1, 1, (n_centres, dim)).astype(np.float32)
    sig = rng.uniform(0.01, 0.2, (n_centres, dim)).astype(np.float32)

    def draw(cnt):
        lab = rng.integers(0, n_centres, cnt)
        return (centres[lab] + sig[lab] * rng.standard_normal((cnt, dim)).astype(np.float32)).astype(np.float32)
    return draw(n), draw(nq)


def _search(idx, q, k, npb, scan, mode=None):
    from vesper_db_b200 import SEARCH_FAST
    old = os.environ.get("VGPU_SCAN")
    if scan is None:
        os.environ.pop("VGPU_SCAN", None)
    else:
        os.environ["VGPU_SCAN"] = scan
    try:
        out = idx.search_batch(q, k, npb, mode=SEARCH_FAST if mode is None else mode)
        return out, idx.last_timings()["scan_variant"]
    finally:
        if old is None:
            os.environ.pop("VGPU_SCAN", None)
        else:
            os.environ["VGPU_SCAN"] = old


SHAPES = {
    # name: dim, m, nlist, n_base, n_train, n_centres, nq, use_opq, searches (k, nprobe)
    "d768_m96_opq": (768, 96, 32, 65536, 20000, 400, 1024, True, [(10, 8), (100, 16)]),
    "d128_m32_dsub4": (128, 32, 64, 98304, 20000, 600, 1024, False, [(100, 16), (10, 4)]),
    "d128_m32_dsub4_opq": (128, 32, 64, 98304, 20000, 600, 1024, True, [(100, 16)]),
}


@pytest.fixture(scope="module", params=list(SHAPES))
def built(request):
    from oracle_lib import read_ivfpq_v10
    from vesper_db_b200 import IvfPqIndex
    dim, m, nlist, n, nt, nc, nq, opq, searches = SHAPES[request.param]
    rng = np.random.default_rng(dim * 7 + m)
    base, q = _mixture(rng, nc, dim, n, nq)
    idx = IvfPqIndex()
    rep = idx.train(base[:nt], nlist, m, 8, use_opq=opq)
    idx.add(np.arange(n, dtype=np.uint64) * 5 + 11, base)
    td = tempfile.mkdtemp(prefix="vesper_headline_")
    idx.save(td)
    f = read_ivfpq_v10(os.path.join(td, "ivfpq.bin"))
    assert (f["rotation"] is not None) == rep.opq_kept
    offs = f["list_offsets"].astype(np.int64)
    sizes = np.diff(offs)
    # the shape this file is about: lists of thousands of entries
    assert sizes.mean() >= 1000, sizes.mean()
    yield dict(name=request.param, idx=idx, f=f, q=q, searches=searches, dir=td, m=m)
    idx.close()
    import shutil
    shutil.rmtree(td, ignore_errors=True)


def _oracle_search(oracle, b, k, npb):
    cache = b.setdefault("oracle_results", {})
    if (k, npb) not in cache:
        f = b["f"]
        cache[(k, npb)] = oracle.ivfpq_search(b["q"], f["centroids"], f["rotation"], f["codebooks"], b["m"],
                                              f["list_offsets"], f["ids"], f["codes"], k, npb)
    return cache[(k, npb)]


def test_exact_mode_bit_exact(built, oracle):
    from vesper_db_b200 import SEARCH_EXACT
    for k, npb in built["searches"]:
        rids, rd, rcnt = _oracle_search(oracle, built, k, npb)
        (ids, d, cnt), _ = _search(built["idx"], built["q"], k, npb, None, mode=SEARCH_EXACT)
        assert np.array_equal(cnt, rcnt)
        for i in range(d.shape[0]):
            assert np.array_equal(d[i, :cnt[i]], rd[i, :rcnt[i]]), (built["name"], k, npb, i)
        assert_topk_equivalent(ids, d, cnt, rids, rd, rcnt, 0.0)


@pytest.mark.parametrize("scan,variant", [("tc", 4), ("blocked", 3)])
def test_fast_mode_within_tolerance(built, oracle, scan, variant):
    for k, npb in built["searches"]:
        rids, rd, rcnt = _oracle_search(oracle, built, k, npb)
        (ids, d, cnt), v = _search(built["idx"], built["q"], k, npb, scan)
        assert v == variant, f"{scan} scan did not run (variant {v})"
        assert_topk_equivalent(ids, d, cnt, rids, rd, rcnt, RTOL)
        rel = np.abs(d.astype(np.float64) - rd) / np.maximum(1.0, np.abs(rd.astype(np.float64)))
        assert rel.max() <= RTOL


def test_list_scan_bit_identical_to_blocked(built):
    for k, npb in built["searches"]:
        (bi, bd, bn), vb = _search(built["idx"], built["q"], k, npb, "blocked")
        (ti, td, tn), vt = _search(built["idx"], built["q"], k, npb, "tc")
        assert (vb, vt) == (3, 4)
        assert np.array_equal(bn, tn) and np.array_equal(bd, td) and np.array_equal(bi, ti)


def test_fast_mode_against_reference_library(built, reference):
    """The same index loaded into the reference's own IvfPqIndex (its v1.0 loader) and
    searched by its search_batch: FAST results within 1e-4 of the reference's."""
    ridx = reference.ivfpq()
    ridx.load(built["dir"])
    nq = 256
    q = built["q"][:nq]
    for k, npb in built["searches"]:
        rids, rd, rcnt = ridx.search(q, k, npb)
        ids, d, cnt = built["idx"].search_batch(q, k, npb)
        assert_topk_equivalent(ids, d, cnt, rids, rd, rcnt, RTOL)
