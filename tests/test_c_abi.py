"""The C-ABI library loads and exports every symbol include/*.h declares (no GPU)."""
import ctypes as C
import os
import re

import pytest

from conftest import ROOT
from vesper_db_b200 import _native as N


def declared_symbols():
    names = set()
    for h in ("vesper.h", "vesper_b200.h"):
        text = open(os.path.join(ROOT, "include", h)).read()
        for mt in re.finditer(r"VESPER_C_API\s+[\w\s\*]+?\b(vesper_\w+)\s*\(", text):
            names.add(mt.group(1))
    return names


def test_library_exports_every_declared_symbol():
    lib = N.load()
    declared = declared_symbols()
    assert len(declared) >= 24
    for name in declared:
        assert hasattr(lib, name), name
    assert declared == set(N.EXPORTED)


def test_reference_symbols_present():
    # Must export the reference's C ABI symbols (include/vesper/c/vesper.h:34-117).
    ref = ["vesper_get_last_error", "vesper_version", "vesper_ivfpq_create", "vesper_ivfpq_destroy",
           "vesper_ivfpq_train", "vesper_ivfpq_add", "vesper_ivfpq_search", "vesper_ivfpq_search_batch",
           "vesper_ivfpq_is_trained", "vesper_ivfpq_get_dimension", "vesper_ivfpq_get_stats",
           "vesper_ivfpq_set_metadata_json", "vesper_ivfpq_get_metadata_json", "vesper_ivfpq_save",
           "vesper_ivfpq_load"]
    lib = N.load()
    for name in ref:
        assert hasattr(lib, name)


def test_null_argument_semantics():
    """NULL arguments -> VESPER_ERROR_INVALID_PARAM without touching a device."""
    lib = N.load()
    assert lib.vesper_version() == b"dev"
    assert lib.vesper_ivfpq_create(None) == N.VESPER_ERROR_INVALID_PARAM
    assert lib.vesper_ivfpq_train(None, None, 0, 0, None) == N.VESPER_ERROR_INVALID_PARAM
    assert lib.vesper_ivfpq_add(None, None, None, 0) == N.VESPER_ERROR_INVALID_PARAM
    assert lib.vesper_ivfpq_search(None, None, None, None, None) == N.VESPER_ERROR_INVALID_PARAM
    assert lib.vesper_ivfpq_search_batch(None, None, 0, None, None, None) == N.VESPER_ERROR_INVALID_PARAM
    assert lib.vesper_ivfpq_is_trained(None, None) == N.VESPER_ERROR_INVALID_PARAM
    assert lib.vesper_ivfpq_get_stats(None, None) == N.VESPER_ERROR_INVALID_PARAM
    assert lib.vesper_ivfpq_save(None, b"/tmp/x") == N.VESPER_ERROR_INVALID_PARAM
    assert lib.vesper_ivfpq_load(None, b"/tmp/x") == N.VESPER_ERROR_INVALID_PARAM
    assert lib.vesper_ivfpq_destroy(None) == N.VESPER_OK
    assert lib.vesper_get_last_error() == b""


def test_train_params_ex_defaults():
    lib = N.load()
    p = N.TrainParamsEx()
    lib.vesper_ivfpq_train_params_ex_init(C.byref(p))
    assert p.struct_size == C.sizeof(N.TrainParamsEx)
    assert (p.nlist, p.m, p.nbits, p.max_iter, p.use_opq, p.opq_iter, p.opq_sample_n, p.seed) == \
        (256, 8, 8, 25, 1, 10, 20000, 42)
    assert abs(p.epsilon - 1e-4) < 1e-9


def test_kmeans_params_and_precondition_errors():
    """kmeans_cluster's checks (src/index/kmeans.cpp:141-151) run before any device work."""
    import numpy as np
    lib = N.load()
    p = N.KmeansParams()
    lib.vesper_kmeans_params_init(C.byref(p))
    assert p.struct_size == C.sizeof(N.KmeansParams)
    assert (p.k, p.max_iter, p.seed, p.algorithm) == (256, 25, 42, N.KMEANS_ELKAN)
    assert abs(p.epsilon - 1e-4) < 1e-9
    x = np.zeros((10, 4), np.float32)
    c = np.zeros((64, 4), np.float32)
    f32 = C.POINTER(C.c_float)
    xp, cp = x.ctypes.data_as(f32), c.ctypes.data_as(f32)
    p.k = 11
    assert lib.vesper_kmeans_fit(xp, 10, 4, C.byref(p), cp, None, None) == N.VESPER_ERROR_INVALID_PARAM
    assert lib.vesper_get_last_error() == b"Not enough data points for k clusters"
    p.k = 0
    assert lib.vesper_kmeans_fit(xp, 10, 4, C.byref(p), cp, None, None) == N.VESPER_ERROR_INVALID_PARAM
    assert lib.vesper_get_last_error() == b"k must be > 0"
    p.k, p.algorithm = 4, 7
    assert lib.vesper_kmeans_fit(xp, 10, 4, C.byref(p), cp, None, None) == N.VESPER_ERROR_INVALID_PARAM
    p.algorithm = N.KMEANS_LLOYD
    assert lib.vesper_kmeans_fit(None, 10, 4, C.byref(p), cp, None, None) == N.VESPER_ERROR_INVALID_PARAM
    assert lib.vesper_kmeans_fit_device(None, 10, 4, C.byref(p), None, None, None) == N.VESPER_ERROR_INVALID_PARAM


def test_flat_topk_precondition_errors():
    """The reference returns early on n_base, nq or k == 0 (batch_distances.hpp:349-350);
    unsupported shapes and operators are rejected before any device work."""
    import numpy as np
    lib = N.load()
    f32, u32 = C.POINTER(C.c_float), C.POINTER(C.c_uint32)
    q = np.zeros((3, 32), np.float32)
    b = np.zeros((10, 32), np.float32)
    i = np.zeros((3, 2000), np.uint32)
    s = np.zeros((3, 2000), np.float32)
    qp, bp, ip, sp = q.ctypes.data_as(f32), b.ctypes.data_as(f32), i.ctypes.data_as(u32), s.ctypes.data_as(f32)
    assert lib.vesper_flat_topk(N.FLAT_L2, qp, 0, bp, 10, 32, 5, ip, sp) == N.VESPER_OK
    assert lib.vesper_flat_topk(N.FLAT_IP, qp, 3, bp, 0, 32, 5, ip, sp) == N.VESPER_OK
    assert lib.vesper_flat_topk(N.FLAT_IP, qp, 3, bp, 10, 32, 0, ip, sp) == N.VESPER_OK
    assert lib.vesper_flat_topk(7, qp, 3, bp, 10, 32, 5, ip, sp) == N.VESPER_ERROR_INVALID_PARAM
    assert lib.vesper_flat_topk(N.FLAT_L2, None, 3, bp, 10, 32, 5, ip, sp) == N.VESPER_ERROR_INVALID_PARAM
    assert lib.vesper_flat_topk(N.FLAT_L2, qp, 3, bp, 10, 32, 1025, ip, sp) == N.VESPER_ERROR_INVALID_PARAM
    assert b"unsupported shape" in lib.vesper_get_last_error()
    assert lib.vesper_flat_topk(N.FLAT_L2, qp, 3, bp, 10, 30, 5, ip, sp) == N.VESPER_ERROR_INVALID_PARAM
    assert lib.vesper_flat_topk_device(N.FLAT_L2, None, 3, None, 10, 32, 5, None, None) == \
        N.VESPER_ERROR_INVALID_PARAM
    t = N.FlatTimings()
    assert lib.vesper_flat_get_last_timings(C.byref(t)) == N.VESPER_OK
    assert lib.vesper_flat_get_last_timings(None) == N.VESPER_ERROR_INVALID_PARAM


def test_missing_library_fails_loudly(tmp_path):
    N_mod = N
    saved = N_mod._lib
    try:
        N_mod._lib = None
        with pytest.raises(RuntimeError, match="missing"):
            N_mod.load(str(tmp_path / "nope.so"))
    finally:
        N_mod._lib = saved
