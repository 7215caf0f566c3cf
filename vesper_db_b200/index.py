"""Python host mirror of the reference's IvfPqIndex over the B200 C ABI.

Method names, argument meaning and error behaviour follow
include/vesper/index/ivf_pq.hpp (train / add / search / search_batch / save / load /
get_stats / is_trained / dimension / set_metadata_json / get_metadata_json); every call
goes through libvesper_c.so, i.e. through the same vesper_ivfpq_* entry points a C
caller of the reference uses.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np

from . import _native as N


class VesperError(RuntimeError):
    """A non-OK vesper_status_t; ``status`` holds the code, the message the last error."""

    def __init__(self, status: int, message: str):
        super().__init__(f"vesper status {status}: {message}")
        self.status = status
        self.message = message


def _check(lib, status: int):
    if status != N.VESPER_OK:
        raise VesperError(status, lib.vesper_get_last_error().decode(errors="replace"))


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def _ptr(a, ctype):
    return a.ctypes.data_as(C.POINTER(ctype))


@dataclass
class TrainReport:
    opq_kept: bool
    err_unrot: float
    err_opq: float
    coarse_iterations: int
    train_time_sec: float


class IvfPqIndex:
    """GPU IVF-PQ index handle (one CUDA device: the current one at creation)."""

    def __init__(self):
        self._lib = N.load()
        if self._lib.vesper_b200_device_count() <= 0:
            raise RuntimeError("no CUDA device visible to libvesper_c.so")
        h = C.c_void_p()
        _check(self._lib, self._lib.vesper_ivfpq_create(C.byref(h)))
        self._h = h

    def close(self):
        if getattr(self, "_h", None):
            self._lib.vesper_ivfpq_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def handle(self):
        return self._h

    # ------------------------------------------------------------------ train / add
    def train(self, data, nlist: int, m: int, nbits: int = 8, *, use_opq: bool = True,
              max_iter: int = 25, epsilon: float = 1e-4, seed: int = 42, opq_iter: int = 10,
              opq_sample_n: int = 20000, opq_init_pca: bool = True, verbose: bool = False) -> TrainReport:
        x = _f32(data)
        p = N.TrainParamsEx()
        self._lib.vesper_ivfpq_train_params_ex_init(C.byref(p))
        p.nlist, p.m, p.nbits = nlist, m, nbits
        p.max_iter, p.epsilon, p.use_opq, p.seed = max_iter, epsilon, int(use_opq), seed
        p.opq_iter, p.opq_sample_n, p.opq_init_pca, p.verbose = opq_iter, opq_sample_n, int(opq_init_pca), int(verbose)
        _check(self._lib, self._lib.vesper_ivfpq_train_ex(self._h, _ptr(x, C.c_float), x.shape[1], x.shape[0],
                                                          C.byref(p)))
        r = N.TrainReport()
        _check(self._lib, self._lib.vesper_ivfpq_get_train_report(self._h, C.byref(r)))
        return TrainReport(bool(r.opq_kept), r.err_unrot, r.err_opq, r.coarse_iterations, r.train_time_sec)

    def train_c(self, data, nlist: int, m: int, nbits: int = 8):
        """vesper_ivfpq_train exactly as a C caller of the reference makes it."""
        x = _f32(data)
        p = N.TrainParams(nlist, m, nbits)
        _check(self._lib, self._lib.vesper_ivfpq_train(self._h, _ptr(x, C.c_float), x.shape[1], x.shape[0],
                                                       C.byref(p)))

    def add(self, ids, data):
        x = _f32(data)
        ids = np.ascontiguousarray(ids, dtype=np.uint64)
        _check(self._lib, self._lib.vesper_ivfpq_add(self._h, _ptr(ids, C.c_uint64), _ptr(x, C.c_float),
                                                     x.shape[0]))

    def train_device(self, x_ptr: int, n: int, dim: int, nlist: int, m: int, nbits: int = 8, *,
                     use_opq: bool = True, max_iter: int = 25, epsilon: float = 1e-4, seed: int = 42,
                     opq_iter: int = 10, opq_sample_n: int = 20000, verbose: bool = False) -> TrainReport:
        """Train from n x dim float32 rows already in device memory (x_ptr)."""
        p = N.TrainParamsEx()
        self._lib.vesper_ivfpq_train_params_ex_init(C.byref(p))
        p.nlist, p.m, p.nbits, p.max_iter, p.epsilon = nlist, m, nbits, max_iter, epsilon
        p.use_opq, p.seed, p.opq_iter, p.opq_sample_n, p.verbose = int(use_opq), seed, opq_iter, opq_sample_n, int(verbose)
        _check(self._lib, self._lib.vesper_ivfpq_train_ex_device(self._h, C.c_void_p(x_ptr), dim, n, C.byref(p)))
        r = N.TrainReport()
        _check(self._lib, self._lib.vesper_ivfpq_get_train_report(self._h, C.byref(r)))
        return TrainReport(bool(r.opq_kept), r.err_unrot, r.err_opq, r.coarse_iterations, r.train_time_sec)

    def add_device(self, ids_ptr: int, x_ptr: int, n: int):
        """Add n vectors whose ids (uint64) and rows (float32) are in device memory."""
        _check(self._lib, self._lib.vesper_ivfpq_add_device(self._h, C.c_void_p(ids_ptr), C.c_void_p(x_ptr), n))

    def set_model(self, centroids, codebooks, rotation=None, nbits: int = 8):
        c, cb = _f32(centroids), _f32(codebooks)
        nlist, dim = c.shape
        dsub = cb.shape[1]
        m = dim // dsub
        R = None if rotation is None else _f32(rotation)
        _check(self._lib, self._lib.vesper_ivfpq_set_model(
            self._h, dim, nlist, m, nbits, _ptr(c, C.c_float), _ptr(cb, C.c_float),
            None if R is None else _ptr(R, C.c_float)))
        self._keep = (c, cb, R)

    # ------------------------------------------------------------------ search
    def search_batch(self, queries, k: int, nprobe: int, mode: int = N.SEARCH_FAST, cand_k: int = 0,
                     use_exact_rerank: bool = False, rerank_k: int = 0):
        """Returns (ids [nq, k] uint64, distances [nq, k] float32, counts [nq] uint32).
        cand_k / use_exact_rerank / rerank_k are IvfPqSearchParams' fields
        (include/vesper/index/ivf_pq.hpp:109-117)."""
        q = _f32(queries)
        nq = q.shape[0]
        ids = np.zeros((nq, k), np.uint64)
        d = np.zeros((nq, k), np.float32)
        cnt = np.zeros(nq, np.uint32)
        p = N.SearchParamsEx(C.sizeof(N.SearchParamsEx), k, nprobe, mode, cand_k, int(use_exact_rerank), rerank_k)
        _check(self._lib, self._lib.vesper_ivfpq_search_batch_ex(
            self._h, _ptr(q, C.c_float), nq, C.byref(p), _ptr(ids, C.c_uint64), _ptr(d, C.c_float),
            _ptr(cnt, C.c_uint32)))
        return ids, d, cnt

    def search_batch_c(self, queries, k: int, nprobe: int):
        """vesper_ivfpq_search_batch exactly as a C caller of the reference makes it."""
        q = _f32(queries)
        nq = q.shape[0]
        ids = np.zeros((nq, k), np.uint64)
        d = np.zeros((nq, k), np.float32)
        p = N.SearchParams(k, nprobe)
        _check(self._lib, self._lib.vesper_ivfpq_search_batch(self._h, _ptr(q, C.c_float), nq, C.byref(p),
                                                              _ptr(ids, C.c_uint64), _ptr(d, C.c_float)))
        return ids, d

    def search(self, query, k: int, nprobe: int):
        q = _f32(query).reshape(-1)
        ids = np.zeros(k, np.uint64)
        d = np.zeros(k, np.float32)
        p = N.SearchParams(k, nprobe)
        _check(self._lib, self._lib.vesper_ivfpq_search(self._h, _ptr(q, C.c_float), C.byref(p),
                                                        _ptr(ids, C.c_uint64), _ptr(d, C.c_float)))
        return ids, d

    def search_batch_device(self, q_ptr: int, nq: int, k: int, nprobe: int, ids_ptr: int, d_ptr: int,
                            counts_ptr: int = 0, mode: int = N.SEARCH_FAST, cand_k: int = 0,
                            use_exact_rerank: bool = False, rerank_k: int = 0):
        """Device-resident search: all pointers are device addresses (e.g. torch data_ptr())."""
        p = N.SearchParamsEx(C.sizeof(N.SearchParamsEx), k, nprobe, mode, cand_k, int(use_exact_rerank), rerank_k)
        _check(self._lib, self._lib.vesper_ivfpq_search_batch_device(
            self._h, C.c_void_p(q_ptr), nq, C.byref(p), C.c_void_p(ids_ptr), C.c_void_p(d_ptr),
            C.c_void_p(counts_ptr) if counts_ptr else None))

    def probe_device(self, q_ptr: int, nq: int, nprobe: int, probe_ptr: int, probe_d_ptr: int):
        """The coarse stage alone: probe lists uint32 [nq, min(nprobe, nlist)] and their
        distances float32 (device addresses)."""
        _check(self._lib, self._lib.vesper_ivfpq_probe_device(self._h, C.c_void_p(q_ptr), nq, nprobe,
                                                              C.c_void_p(probe_ptr), C.c_void_p(probe_d_ptr)))

    def search_batch_device_probed(self, q_ptr: int, nq: int, k: int, nprobe: int, probe_ptr: int,
                                   probe_d_ptr: int, ids_ptr: int, d_ptr: int, counts_ptr: int = 0,
                                   mode: int = N.SEARCH_FAST):
        """search_batch_device with the probe lists given (as probe_device writes them)."""
        p = N.SearchParamsEx(C.sizeof(N.SearchParamsEx), k, nprobe, mode, 0, 0, 0)
        _check(self._lib, self._lib.vesper_ivfpq_search_batch_device_probed(
            self._h, C.c_void_p(q_ptr), nq, C.byref(p), C.c_void_p(probe_ptr), C.c_void_p(probe_d_ptr),
            C.c_void_p(ids_ptr), C.c_void_p(d_ptr), C.c_void_p(counts_ptr) if counts_ptr else None))

    def set_threshold_exchange(self, fn, shard: int = 0, shards: int = 1):
        """Install fn(d_tau, n_queries, cuda_stream, user) -> int (an N.TAU_EXCHANGE_FN
        object, kept alive here) as the index's threshold exchange between shards, or
        remove it with None (vesper_ivfpq_set_threshold_exchange).  With shards > 1 this
        index bounds only the queries q with q % shards == shard itself."""
        cb = fn if fn is None or isinstance(fn, N.TAU_EXCHANGE_FN) else N.TAU_EXCHANGE_FN(fn)
        _check(self._lib, self._lib.vesper_ivfpq_set_threshold_exchange(
            self._h, cb if cb is not None else N.TAU_EXCHANGE_FN(), None, shard if cb is not None else 0,
            shards if cb is not None else 1))
        self._tau_cb = cb

    # ------------------------------------------------------------------ the rest of the index API
    # (IvfPqIndex::reconstruct & co., include/vesper/index/ivf_pq.hpp:252-386)
    def reconstruct(self, vid: int) -> np.ndarray:
        out = np.zeros(self.dimension(), np.float32)
        _check(self._lib, self._lib.vesper_ivfpq_reconstruct(self._h, vid, _ptr(out, C.c_float)))
        return out

    get_vector = reconstruct

    def reconstruct_cluster(self, cluster_id: int):
        """(ids uint64 [n], vectors float32 [n, dim]) of the cluster, list order."""
        n = C.c_size_t(0)
        st = self._lib.vesper_ivfpq_reconstruct_cluster(self._h, cluster_id, None, None, 0, C.byref(n))
        if st != N.VESPER_OK and n.value == 0:
            _check(self._lib, st)  # an error other than the capacity probe
        dim = self.dimension()
        ids = np.zeros(max(1, n.value), np.uint64)
        vec = np.zeros(max(1, n.value) * dim, np.float32)
        _check(self._lib, self._lib.vesper_ivfpq_reconstruct_cluster(self._h, cluster_id, _ptr(ids, C.c_uint64),
                                                                     _ptr(vec, C.c_float), ids.shape[0], C.byref(n)))
        return ids[:n.value], vec[:n.value * dim].reshape(n.value, dim)

    def get_cluster_assignment(self, vid: int) -> int:
        out = C.c_uint32(0)
        _check(self._lib, self._lib.vesper_ivfpq_get_cluster_assignment(self._h, vid, C.byref(out)))
        return out.value

    def get_cluster_centroid(self, cluster_id: int) -> np.ndarray:
        out = np.zeros(self.dimension(), np.float32)
        _check(self._lib, self._lib.vesper_ivfpq_get_cluster_centroid(self._h, cluster_id, _ptr(out, C.c_float)))
        return out

    def update_cluster_centroid(self, cluster_id: int, centroid):
        c = _f32(centroid)
        _check(self._lib, self._lib.vesper_ivfpq_update_cluster_centroid(self._h, cluster_id, _ptr(c, C.c_float)))

    def reassign_vector(self, vid: int, new_cluster: int):
        _check(self._lib, self._lib.vesper_ivfpq_reassign_vector(self._h, vid, new_cluster))

    def compact_inverted_list(self, cluster_id: int, deleted_ids) -> int:
        d = np.ascontiguousarray(deleted_ids, np.uint32)
        out = C.c_size_t(0)
        _check(self._lib, self._lib.vesper_ivfpq_compact_inverted_list(self._h, cluster_id, _ptr(d, C.c_uint32),
                                                                       d.shape[0], C.byref(out)))
        return out.value

    def debug_explain_centroid_rank(self, query, vid: int):
        q = _f32(query).reshape(-1)
        rank, cl = C.c_uint64(0), C.c_uint32(0)
        _check(self._lib, self._lib.vesper_ivfpq_debug_explain_centroid_rank(self._h, _ptr(q, C.c_float), vid,
                                                                             C.byref(rank), C.byref(cl)))
        return rank.value, cl.value

    def debug_explain_adc_rank(self, query, vid: int):
        q = _f32(query).reshape(-1)
        rank, d = C.c_uint64(0), C.c_float(0)
        _check(self._lib, self._lib.vesper_ivfpq_debug_explain_adc_rank(self._h, _ptr(q, C.c_float), vid,
                                                                        C.byref(rank), C.byref(d)))
        return rank.value, d.value

    def search_batch_device_noalloc(self, q_ptr: int, nq: int, k: int, nprobe: int, ids_ptr: int, d_ptr: int,
                                    counts_ptr: int = 0):
        """Like search_batch_device (FAST mode) but allocating nothing: temporaries live in
        the library's fixed 64 MiB device array (see include/vesper_b200.h)."""
        p = N.SearchParamsEx(C.sizeof(N.SearchParamsEx), k, nprobe, N.SEARCH_FAST)
        _check(self._lib, self._lib.vesper_ivfpq_search_batch_device_noalloc(
            self._h, C.c_void_p(q_ptr), nq, C.byref(p), C.c_void_p(ids_ptr), C.c_void_p(d_ptr),
            C.c_void_p(counts_ptr) if counts_ptr else None))

    def last_timings(self) -> dict:
        t = N.Timings()
        _check(self._lib, self._lib.vesper_ivfpq_get_last_timings(self._h, C.byref(t)))
        return {f: getattr(t, f) for f, _ in N.Timings._fields_}

    # ------------------------------------------------------------------ state
    def is_trained(self) -> bool:
        v = C.c_int()
        _check(self._lib, self._lib.vesper_ivfpq_is_trained(self._h, C.byref(v)))
        return bool(v.value)

    def dimension(self) -> int:
        v = C.c_size_t()
        _check(self._lib, self._lib.vesper_ivfpq_get_dimension(self._h, C.byref(v)))
        return v.value

    def get_stats(self) -> dict:
        s = N.Stats()
        _check(self._lib, self._lib.vesper_ivfpq_get_stats(self._h, C.byref(s)))
        return {f: getattr(s, f) for f, _ in N.Stats._fields_}

    def list_offsets(self) -> np.ndarray:
        """CSR offsets [nlist+1] of the inverted lists (list l holds entries offs[l]..offs[l+1])."""
        offs = np.zeros(self.get_stats()["n_lists"] + 1, np.uint64)
        _check(self._lib, self._lib.vesper_ivfpq_get_lists(self._h, _ptr(offs, C.c_uint64), None, None))
        return offs

    def lists(self):
        """(offsets [nlist+1], ids [N], codes [N, m]) copied from the device."""
        st = self.get_stats()
        nlist, n, m = st["n_lists"], st["n_vectors"], st["m"]
        offs = np.zeros(nlist + 1, np.uint64)
        ids = np.zeros(max(n, 1), np.uint64)
        codes = np.zeros((max(n, 1), m), np.uint8)
        _check(self._lib, self._lib.vesper_ivfpq_get_lists(self._h, _ptr(offs, C.c_uint64), _ptr(ids, C.c_uint64),
                                                           _ptr(codes, C.c_uint8)))
        return offs, ids[:n], codes[:n]

    def set_metadata_json(self, s: str):
        _check(self._lib, self._lib.vesper_ivfpq_set_metadata_json(self._h, s.encode()))

    def get_metadata_json(self) -> str:
        need = C.c_size_t()
        _check(self._lib, self._lib.vesper_ivfpq_get_metadata_json(self._h, None, 0, C.byref(need)))
        buf = C.create_string_buffer(need.value)
        _check(self._lib, self._lib.vesper_ivfpq_get_metadata_json(self._h, buf, need.value, C.byref(need)))
        return buf.value.decode()

    def save(self, directory: str):
        _check(self._lib, self._lib.vesper_ivfpq_save(self._h, directory.encode()))

    def load(self, directory: str):
        _check(self._lib, self._lib.vesper_ivfpq_load(self._h, directory.encode()))

    @classmethod
    def from_file(cls, directory: str) -> "IvfPqIndex":
        idx = cls()
        idx.load(directory)
        return idx
