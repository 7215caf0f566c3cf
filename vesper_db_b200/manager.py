"""Python mirror of the reference's IndexManager C ABI (include/vesper/c/vesper_manager.h)
over libvesper_c.so: the manager routes IVF-PQ builds, updates, removals and searches to
the GPU index (include/vesper_manager.h states what it keeps from the reference and what
it refuses).  Every call raises VesperError with the library's message on failure."""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import _native as N
from .index import _check, _f32, _ptr


def query_config(k: int = 10, nprobe: int = 8, use_exact_rerank: bool = False, rerank_k: int = 0,
                 rerank_alpha: float = 2.0, rerank_cand_ceiling: int = 2000, preferred_index=None,
                 filter_json: str | None = None) -> N.QueryConfig:
    """A vesper_query_config_t with the reference's QueryConfig defaults
    (include/vesper/index/index_manager.hpp:79-101)."""
    qc = N.QueryConfig()
    qc.k, qc.epsilon, qc.ef_search, qc.nprobe, qc.l_search = k, 0.0, 100, nprobe, 128
    qc.use_exact_rerank, qc.rerank_k = int(use_exact_rerank), rerank_k
    qc.rerank_alpha, qc.rerank_cand_ceiling, qc.use_query_planner = rerank_alpha, rerank_cand_ceiling, 1
    qc.has_preferred_index = int(preferred_index is not None)
    qc.preferred_index = preferred_index if preferred_index is not None else 0
    qc.has_filter = int(filter_json is not None)
    qc.filter_json = filter_json.encode() if filter_json is not None else None
    return qc


class IndexManager:
    """vesper_mgr_* over one manager handle."""

    def __init__(self, dim: int):
        self._lib = N.load()
        self._h = C.c_void_p()
        self.dim = dim
        _check(self._lib, self._lib.vesper_mgr_create(dim, C.byref(self._h)))

    def close(self):
        if self._h:
            self._lib.vesper_mgr_destroy(self._h)
            self._h = None

    def __del__(self):
        self.close()

    def build(self, x, index_type: int = N.INDEX_IVF_PQ, strategy: int = N.SELECT_MANUAL, nlist: int = 0,
              m: int = 0, nbits: int = 8):
        x = _f32(x)
        cfg = N.ManagerBuildConfig()
        cfg.type, cfg.strategy = index_type, strategy
        cfg.ivf.nlist, cfg.ivf.m, cfg.ivf.nbits = nlist, m, nbits
        cfg.hnsw.M, cfg.hnsw.ef_construction, cfg.hnsw.seed = 16, 200, 42
        cfg.vamana.degree, cfg.vamana.L, cfg.vamana.alpha = 64, 128, 1.2
        _check(self._lib, self._lib.vesper_mgr_build(self._h, _ptr(x, C.c_float), x.shape[0], C.byref(cfg)))

    def add_batch(self, ids, x):
        ids = np.ascontiguousarray(ids, np.uint64)
        x = _f32(x)
        _check(self._lib, self._lib.vesper_mgr_add_batch(self._h, _ptr(ids, C.c_uint64), _ptr(x, C.c_float),
                                                         x.shape[0]))

    def update(self, vid: int, v):
        v = _f32(v)
        _check(self._lib, self._lib.vesper_mgr_update(self._h, vid, _ptr(v, C.c_float)))

    def update_batch(self, ids, x):
        ids = np.ascontiguousarray(ids, np.uint64)
        x = _f32(x)
        _check(self._lib, self._lib.vesper_mgr_update_batch(self._h, _ptr(ids, C.c_uint64), _ptr(x, C.c_float),
                                                            x.shape[0]))

    def remove(self, vid: int):
        _check(self._lib, self._lib.vesper_mgr_remove(self._h, vid))

    def remove_batch(self, ids):
        ids = np.ascontiguousarray(ids, np.uint64)
        _check(self._lib, self._lib.vesper_mgr_remove_batch(self._h, _ptr(ids, C.c_uint64), ids.shape[0]))

    def search(self, q, qc: N.QueryConfig):
        q = _f32(q).reshape(1, -1)
        return self.search_batch(q, qc, single=True)

    def search_batch(self, queries, qc: N.QueryConfig, single: bool = False):
        q = _f32(queries)
        nq = q.shape[0]
        ids = np.zeros((nq, qc.k), np.uint64)
        d = np.zeros((nq, qc.k), np.float32)
        if single:
            _check(self._lib, self._lib.vesper_mgr_search(self._h, _ptr(q, C.c_float), C.byref(qc),
                                                          _ptr(ids, C.c_uint64), _ptr(d, C.c_float)))
        else:
            _check(self._lib, self._lib.vesper_mgr_search_batch(self._h, _ptr(q, C.c_float), nq, C.byref(qc),
                                                                _ptr(ids, C.c_uint64), _ptr(d, C.c_float)))
        return ids, d

    def save(self, directory: str):
        _check(self._lib, self._lib.vesper_mgr_save(self._h, directory.encode()))

    def load(self, directory: str):
        _check(self._lib, self._lib.vesper_mgr_load(self._h, directory.encode()))

    def memory_usage(self) -> int:
        v = C.c_size_t(0)
        _check(self._lib, self._lib.vesper_mgr_memory_usage(self._h, C.byref(v)))
        return int(v.value)

    def disk_usage(self) -> int:
        v = C.c_size_t(0)
        _check(self._lib, self._lib.vesper_mgr_disk_usage(self._h, C.byref(v)))
        return int(v.value)

    def set_memory_budget_mb(self, mb: int):
        _check(self._lib, self._lib.vesper_mgr_set_memory_budget_mb(self._h, mb))

    def get_memory_budget_mb(self) -> int:
        v = C.c_uint32(0)
        _check(self._lib, self._lib.vesper_mgr_get_memory_budget_mb(self._h, C.byref(v)))
        return int(v.value)

    def get_stats(self) -> list[dict]:
        cnt = C.c_size_t(0)
        _check(self._lib, self._lib.vesper_mgr_get_stats(self._h, None, None, C.byref(cnt)))
        n = cnt.value
        arr = (N.IndexStats * max(n, 1))()
        cap = C.c_size_t(n)
        _check(self._lib, self._lib.vesper_mgr_get_stats(self._h, arr, C.byref(cap), C.byref(cnt)))
        return [{f: getattr(arr[i], f) for f, _ in N.IndexStats._fields_} for i in range(n)]

    def set_search_mode(self, mode: int):
        _check(self._lib, self._lib.vesper_mgr_set_search_mode(self._h, mode))
