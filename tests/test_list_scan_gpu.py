"""Tensor-core list scan (FAST mode, VGPU_SCAN=tc) against the blocked scan.

The list scan screens (query, entry) pairs with bf16 tcgen05 products and re-scores the
survivors with the blocked scan's own arithmetic and scan positions, so its results
must equal the blocked scan's bit for bit: ids, distances and counts.  The cases cover
every supported sub-vector width (dim / m = 4, 8, 16), both accumulator widths (N = 128
for dim <= 512, N = 64 above), OPQ rotations, ragged 128-entry tiles, queries whose
nearest list holds fewer than k entries (not screened), candidate-list overflow (the
blocked-scan fallback), and exact ties (duplicated vectors).
"""
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _index():
    from vesper_db_b200 import IvfPqIndex
    return IvfPqIndex()


def _search(idx, q, k, npb, scan, threshold=None, cta=None, refine_table_min=None):
    env = {"VGPU_SCAN": scan, "VGPU_LIST_THRESHOLD": threshold, "VGPU_LIST_CTA": cta,
           "VGPU_REFINE_TABLE_MIN": refine_table_min}
    old = {key: os.environ.get(key) for key in env}
    for key, val in env.items():
        if val is None:
            os.environ.pop(key, None)
        else:
            os.environ[key] = val
    try:
        out = idx.search_batch(q, k, npb)
        variant = idx.last_timings()["scan_variant"]
    finally:
        for key, val in old.items():
            if val is None:
                os.environ.pop(key, None)
            else:
                os.environ[key] = val
    return out, variant


def _build(rng, dim, m, nlist, n, rot, sigma=0.3, dup=0):
    cent = rng.standard_normal((nlist, dim)).astype(np.float32)
    cb = (0.3 * rng.standard_normal((m * 256, dim // m))).astype(np.float32)
    R = np.linalg.qr(rng.standard_normal((dim, dim)))[0].astype(np.float32) if rot else None
    base = (cent[rng.integers(0, nlist, n)] + sigma * rng.standard_normal((n, dim))).astype(np.float32)
    if dup:
        base[-dup:] = base[:dup]
    idx = _index()
    idx.set_model(cent, cb, R)
    idx.add(np.arange(n, dtype=np.uint64) * 7 + 3, base)
    return idx, cent


CASES = [
    # dim, m, nlist, n, nq, rot, searches (k, nprobe)
    (128, 16, 64, 40000, 300, False, [(10, 8), (100, 16), (1, 2)]),
    (128, 32, 64, 40000, 300, True, [(10, 8), (50, 33)]),
    (256, 16, 32, 30000, 200, True, [(10, 6), (100, 12)]),
    (768, 96, 48, 20000, 130, True, [(10, 8), (100, 20)]),
    (512, 64, 40, 20000, 150, False, [(20, 10)]),
    (128, 16, 6, 90000, 300, True, [(10, 3), (100, 5)]),   # nearest lists > 8192 entries
]


@pytest.mark.parametrize("threshold", [None, "tc"])
@pytest.mark.parametrize("dim,m,nlist,n,nq,rot,searches", CASES)
def test_list_scan_equals_blocked_scan(dim, m, nlist, n, nq, rot, searches, threshold):
    """threshold None: long nearest lists get their threshold from the tensor-core
    pass, short ones from the blocked scan; "tc": every query from the tensor cores."""
    rng = np.random.default_rng(dim + m + nlist)
    idx, cent = _build(rng, dim, m, nlist, n, rot)
    q = (cent[rng.integers(0, nlist, nq)] + 0.3 * rng.standard_normal((nq, dim))).astype(np.float32)
    for k, npb in searches:
        (bi, bd, bn), vb = _search(idx, q, k, npb, "blocked")
        (ti, td, tn), vt = _search(idx, q, k, npb, "tc", threshold)
        assert vb == 3 and vt == 4
        assert np.array_equal(bn, tn)
        assert np.array_equal(bd, td)
        assert np.array_equal(bi, ti)


@pytest.mark.parametrize("table_min", ["0", "1000000"])
@pytest.mark.parametrize("dim,m,nlist,n,nq,rot,searches", CASES)
def test_refine_paths_equal_blocked_scan(dim, m, nlist, n, nq, rot, searches, table_min):
    """The refine reads a query's lookup table when it has many candidates and computes
    its candidates' table entries from the rotated query and the codebook otherwise;
    forced to either path for every query, the results stay the blocked scan's."""
    rng = np.random.default_rng(dim + m + nlist)
    idx, cent = _build(rng, dim, m, nlist, n, rot)
    q = (cent[rng.integers(0, nlist, nq)] + 0.3 * rng.standard_normal((nq, dim))).astype(np.float32)
    for k, npb in searches:
        (bi, bd, bn), _ = _search(idx, q, k, npb, "blocked")
        (ti, td, tn), vt = _search(idx, q, k, npb, "tc", refine_table_min=table_min)
        assert vt == 4
        assert np.array_equal(bn, tn) and np.array_equal(bd, td) and np.array_equal(bi, ti)


@pytest.mark.parametrize("dim,m,nlist,n,nq,rot,searches", CASES)
def test_cta_pair_screen_equals_blocked_scan(dim, m, nlist, n, nq, rot, searches):
    """The screen on CTA pairs (tcgen05 cta_group::2, M = 256: two tiles per unit, the
    query tile split between the two SMs) keeps the same pairs: bit-identical results."""
    rng = np.random.default_rng(dim + m + nlist)
    idx, cent = _build(rng, dim, m, nlist, n, rot)
    q = (cent[rng.integers(0, nlist, nq)] + 0.3 * rng.standard_normal((nq, dim))).astype(np.float32)
    for k, npb in searches:
        (bi, bd, bn), _ = _search(idx, q, k, npb, "blocked")
        for threshold in (None, "tc"):
            (ti, td, tn), vt = _search(idx, q, k, npb, "tc", threshold, cta="2")
            assert vt == 4
            assert np.array_equal(bn, tn) and np.array_equal(bd, td) and np.array_equal(bi, ti)


@pytest.mark.parametrize("dim,m,nlist,n,nq,rot,searches", CASES[:2])
def test_split_scan_equals_blocked_scan(dim, m, nlist, n, nq, rot, searches):
    """The blocked scan with each query's blocks split over several CTAs and merged
    (used for the list scan's thresholds and overflow fallback) is bit-identical."""
    rng = np.random.default_rng(dim + m + nlist)
    idx, cent = _build(rng, dim, m, nlist, n, rot)
    q = (cent[rng.integers(0, nlist, nq)] + 0.3 * rng.standard_normal((nq, dim))).astype(np.float32)
    for k, npb in searches + [(1000, 40)]:
        (bi, bd, bn), _ = _search(idx, q, k, npb, "blocked")
        (si, sd, sn), vs = _search(idx, q, k, npb, "split")
        assert vs == 3
        assert np.array_equal(bn, sn) and np.array_equal(bd, sd) and np.array_equal(bi, si)


def test_small_home_lists_and_overflow():
    """Many lists smaller than k (those queries skip the screen), and k large enough that
    some candidate lists overflow (the blocked scan takes those queries over)."""
    rng = np.random.default_rng(77)
    dim, m = 128, 16
    idx, cent = _build(rng, dim, m, 300, 12000, True, sigma=0.05)
    q = (cent[rng.integers(0, 300, 200)] + 0.05 * rng.standard_normal((200, dim))).astype(np.float32)
    for k, npb in [(100, 10), (1000, 40), (64, 300)]:
        (bi, bd, bn), _ = _search(idx, q, k, npb, "blocked")
        (ti, td, tn), vt = _search(idx, q, k, npb, "tc")
        assert vt == 4
        assert np.array_equal(bn, tn) and np.array_equal(bd, td) and np.array_equal(bi, ti)


def test_exact_ties_keep_scan_order():
    rng = np.random.default_rng(5)
    idx, cent = _build(rng, 128, 16, 32, 20000, False, dup=6000)
    q = (cent[rng.integers(0, 32, 256)] + 0.3 * rng.standard_normal((256, 128))).astype(np.float32)
    for k, npb in [(10, 4), (200, 8)]:
        (bi, bd, bn), _ = _search(idx, q, k, npb, "blocked")
        (ti, td, tn), _ = _search(idx, q, k, npb, "tc")
        assert np.array_equal(bn, tn) and np.array_equal(bd, td) and np.array_equal(bi, ti)


@pytest.mark.parametrize("dim,m", [(128, 16), (128, 32), (256, 64), (64, 16), (96, 24), (256, 16), (64, 32), (256, 32)])
def test_register_lut_equals_generic_lut(dim, m):
    """The register-resident table kernel (thread-fixed entries) writes the same tables
    as the generic one: FAST searches through both are bit-identical (dsub = dim / m in
    {2, 4, 8, 16}, sub-space groups of 4 to 32)."""
    rng = np.random.default_rng(dim + m)
    idx, cent = _build(rng, dim, m, 32, 6000, True)
    q = (cent[rng.integers(0, 32, 70)] + 0.3 * rng.standard_normal((70, dim))).astype(np.float32)
    a, _ = _search(idx, q, 10, 4, "blocked")
    os.environ["VGPU_LUT_GENERIC"] = "1"
    try:
        b, _ = _search(idx, q, 10, 4, "blocked")
    finally:
        os.environ.pop("VGPU_LUT_GENERIC", None)
    for x, y in zip(a, b):
        assert np.array_equal(x, y)
