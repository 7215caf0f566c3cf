"""The C-ABI library loads and exports every symbol include/*.h declares (no GPU)."""
import ctypes as C
import os
import re

import numpy as np

import pytest

from conftest import ROOT
from vesper_db_b200 import _native as N


def declared_symbols():
    names = set()
    for h in ("vesper.h", "vesper_b200.h", "vesper_manager.h"):
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


def test_manager_symbols_present():
    # The reference's IndexManager C ABI (include/vesper/c/vesper_manager.h:79-117).
    ref = ["vesper_mgr_create", "vesper_mgr_destroy", "vesper_mgr_build", "vesper_mgr_add_batch",
           "vesper_mgr_update", "vesper_mgr_update_batch", "vesper_mgr_remove", "vesper_mgr_remove_batch",
           "vesper_mgr_search", "vesper_mgr_search_batch", "vesper_mgr_save", "vesper_mgr_load",
           "vesper_mgr_memory_usage", "vesper_mgr_disk_usage", "vesper_mgr_set_memory_budget_mb",
           "vesper_mgr_get_memory_budget_mb", "vesper_mgr_get_stats"]
    lib = N.load()
    for name in ref:
        assert hasattr(lib, name)


def test_manager_host_logic_without_index():
    """Entry points that need no GPU index: create, budget, stats, removal bookkeeping,
    search refusal, and a save/load round trip of the manifest and tombstones (the
    manager holds no IVF-PQ index, so nothing touches a device)."""
    import ctypes as C
    import tempfile
    lib = N.load()
    h = C.c_void_p()
    assert lib.vesper_mgr_create(0, C.byref(h)) == N.VESPER_ERROR_INVALID_PARAM
    assert lib.vesper_mgr_create(16, C.byref(h)) == N.VESPER_OK
    try:
        mb = C.c_uint32(0)
        assert lib.vesper_mgr_get_memory_budget_mb(h, C.byref(mb)) == N.VESPER_OK and mb.value == 1024
        assert lib.vesper_mgr_set_memory_budget_mb(h, 77) == N.VESPER_OK
        lib.vesper_mgr_get_memory_budget_mb(h, C.byref(mb))
        assert mb.value == 77
        cnt = C.c_size_t(5)
        assert lib.vesper_mgr_get_stats(h, None, None, C.byref(cnt)) == N.VESPER_OK and cnt.value == 0
        for vid in (3, 70000, 2**32 + 5, 123456789):
            assert lib.vesper_mgr_remove(h, vid) == N.VESPER_OK
        assert lib.vesper_mgr_remove(h, 3) == N.VESPER_ERROR_INVALID_PARAM
        assert b"already marked" in lib.vesper_get_last_error()
        # 5000 ids in one 64K block: a bitset container
        ids = np.arange(200000, 205000, dtype=np.uint64)
        assert lib.vesper_mgr_remove_batch(h, ids.ctypes.data_as(C.POINTER(C.c_uint64)), ids.size) == N.VESPER_OK
        q = np.zeros(16, np.float32)
        qc = N.QueryConfig()
        qc.k = 5
        out_i = np.zeros(5, np.uint64)
        out_d = np.zeros(5, np.float32)
        rc = lib.vesper_mgr_search(h, q.ctypes.data_as(C.POINTER(C.c_float)), C.byref(qc),
                                   out_i.ctypes.data_as(C.POINTER(C.c_uint64)),
                                   out_d.ctypes.data_as(C.POINTER(C.c_float)))
        assert rc == N.VESPER_ERROR_INVALID_PARAM and b"No suitable index" in lib.vesper_get_last_error()
        with tempfile.TemporaryDirectory() as td:
            assert lib.vesper_mgr_save(h, td.encode()) == N.VESPER_OK
            raw = open(os.path.join(td, "index_manager.manifest"), "rb").read()
            # u32 version, u64 dim, u64 total, u64 budget, bool, i32 strategy, i32 type,
            # u64 budget, u64 cache, 3 x u32 hnsw, 3 x u32 ivf, u32 + f32 + u32 vamana, 3 x bool
            assert len(raw) == 4 + 8 * 3 + 1 + 4 + 4 + 8 + 8 + 12 + 12 + 12 + 3
            assert int.from_bytes(raw[4:12], "little") == 16 and int.from_bytes(raw[20:28], "little") == 77
            h2 = C.c_void_p()
            assert lib.vesper_mgr_create(4, C.byref(h2)) == N.VESPER_OK
            try:
                assert lib.vesper_mgr_load(h2, td.encode()) == N.VESPER_OK
                # the tombstones came back: removing any of them again is refused
                for vid in (3, 70000, 5, 123456789, 200000, 204999):
                    assert lib.vesper_mgr_remove(h2, vid) == N.VESPER_ERROR_INVALID_PARAM, vid
                assert lib.vesper_mgr_remove(h2, 205000) == N.VESPER_OK
            finally:
                lib.vesper_mgr_destroy(h2)
    finally:
        lib.vesper_mgr_destroy(h)


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
