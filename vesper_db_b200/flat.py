"""Python mirror of the reference's exact flat top-k over the B200 C ABI.

`find_nearest_centroids_batch_fused` (include/vesper/kernels/batch_distances.hpp:338-456):
for each query the k_eff = min(k, n_base) best base rows -- squared L2 ascending or
inner product descending, scores in the reference's AVX2 lane order, ties to the smaller
index.  `flat_topk` takes host arrays (vesper_flat_topk), `flat_topk_device` device
addresses (vesper_flat_topk_device).  Entries past k_eff (k > n_base) hold index
0xffffffff and the worst score.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import _native as N
from .index import VesperError, _check, _f32, _ptr

L2 = N.FLAT_L2
INNER_PRODUCT = N.FLAT_IP


def _op(op) -> int:
    if op in (L2, "l2", "L2"):
        return L2
    if op in (INNER_PRODUCT, "ip", "inner_product", "InnerProduct"):
        return INNER_PRODUCT
    raise VesperError(N.VESPER_ERROR_INVALID_PARAM, f"unknown distance op {op!r}")


def flat_topk(op, queries, base, k: int) -> tuple[np.ndarray, np.ndarray]:
    """Returns (indices uint32 [nq, k], scores float32 [nq, k])."""
    q, b = _f32(queries), _f32(base)
    if q.ndim != 2 or b.ndim != 2 or q.shape[1] != b.shape[1]:
        raise VesperError(N.VESPER_ERROR_INVALID_PARAM, "queries [nq, dim] and base [n, dim] expected")
    lib = N.load()
    idx = np.zeros((q.shape[0], k), np.uint32)
    sc = np.zeros((q.shape[0], k), np.float32)
    _check(lib, lib.vesper_flat_topk(_op(op), _ptr(q, C.c_float), q.shape[0], _ptr(b, C.c_float), b.shape[0],
                                     q.shape[1], k, _ptr(idx, C.c_uint32), _ptr(sc, C.c_float)))
    return idx, sc


def flat_topk_device(op, q_ptr: int, nq: int, base_ptr: int, n_base: int, dim: int, k: int, idx_ptr: int,
                     score_ptr: int) -> None:
    """Device-resident call: queries [nq, dim] f32, base [n_base, dim] f32, indices
    [nq, k] u32 and scores [nq, k] f32 at device addresses (e.g. torch data_ptr())."""
    lib = N.load()
    _check(lib, lib.vesper_flat_topk_device(_op(op), C.c_void_p(q_ptr), nq, C.c_void_p(base_ptr), n_base, dim, k,
                                            C.c_void_p(idx_ptr), C.c_void_p(score_ptr)))


def last_timings() -> dict:
    """Stage times (ms) and counters of this thread's last flat top-k call."""
    lib = N.load()
    t = N.FlatTimings()
    _check(lib, lib.vesper_flat_get_last_timings(C.byref(t)))
    return {name: getattr(t, name) for name, _ in N.FlatTimings._fields_}
