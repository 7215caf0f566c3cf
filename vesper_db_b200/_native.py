"""ctypes binding of libvesper_c.so (include/vesper.h + include/vesper_b200.h).

The library is built in-tree by vesper_db_b200/build.py.  There is no fallback: if
the shared library is missing, loading raises instead of silently using anything else.
"""
from __future__ import annotations

import ctypes as C
import os
import threading

PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG, "libvesper_c.so")

VESPER_OK = 0
VESPER_ERROR_UNKNOWN = 1
VESPER_ERROR_INVALID_PARAM = 2
VESPER_ERROR_NOT_TRAINED = 3
VESPER_ERROR_IO = 4
VESPER_ERROR_INTERNAL = 5

SEARCH_FAST = 0
SEARCH_EXACT = 1

# Every symbol the headers in include/ declare.
EXPORTED = [
    "vesper_get_last_error", "vesper_version", "vesper_ivfpq_create", "vesper_ivfpq_destroy",
    "vesper_ivfpq_train", "vesper_ivfpq_add", "vesper_ivfpq_search", "vesper_ivfpq_search_batch",
    "vesper_ivfpq_is_trained", "vesper_ivfpq_get_dimension", "vesper_ivfpq_get_stats",
    "vesper_ivfpq_set_metadata_json", "vesper_ivfpq_get_metadata_json", "vesper_ivfpq_save",
    "vesper_ivfpq_load",
    "vesper_ivfpq_train_params_ex_init", "vesper_ivfpq_train_ex", "vesper_ivfpq_get_train_report",
    "vesper_ivfpq_search_batch_ex", "vesper_ivfpq_search_batch_device", "vesper_ivfpq_get_last_timings",
    "vesper_ivfpq_set_model", "vesper_ivfpq_get_lists", "vesper_b200_device_count",
    "vesper_ivfpq_train_ex_device", "vesper_ivfpq_add_device",
    "vesper_ivfpq_search_batch_device_noalloc",
    "vesper_kmeans_params_init", "vesper_kmeans_fit", "vesper_kmeans_fit_device",
    "vesper_flat_topk", "vesper_flat_topk_device", "vesper_flat_get_last_timings",
    "vesper_ivfpq_probe_device", "vesper_ivfpq_search_batch_device_probed",
    "vesper_ivfpq_set_threshold_exchange", "vesper_topk_merge_device",
    "vesper_ivfpq_reconstruct", "vesper_ivfpq_reconstruct_cluster", "vesper_ivfpq_get_cluster_assignment",
    "vesper_ivfpq_get_cluster_centroid", "vesper_ivfpq_update_cluster_centroid", "vesper_ivfpq_reassign_vector",
    "vesper_ivfpq_compact_inverted_list", "vesper_ivfpq_debug_explain_centroid_rank",
    "vesper_ivfpq_debug_explain_adc_rank",
    "vesper_kmeans_shard_create", "vesper_kmeans_shard_destroy", "vesper_kmeans_shard_assign",
    "vesper_kmeans_shard_pp_update", "vesper_kmeans_shard_accumulate", "vesper_kmeans_shard_finish",
    "vesper_kmeans_shard_running_inertia", "vesper_kmeanspp_sampler_create", "vesper_kmeanspp_sampler_next",
    "vesper_kmeanspp_sampler_destroy",
    "vesper_mgr_create", "vesper_mgr_destroy", "vesper_mgr_build", "vesper_mgr_add_batch", "vesper_mgr_update",
    "vesper_mgr_update_batch", "vesper_mgr_remove", "vesper_mgr_remove_batch", "vesper_mgr_search",
    "vesper_mgr_search_batch", "vesper_mgr_save", "vesper_mgr_load", "vesper_mgr_memory_usage",
    "vesper_mgr_disk_usage", "vesper_mgr_set_memory_budget_mb", "vesper_mgr_get_memory_budget_mb",
    "vesper_mgr_get_stats", "vesper_mgr_set_search_mode",
]

# int fn(float* d_tau, size_t n_queries, void* cuda_stream, void* user)
# (vesper_ivfpq_set_threshold_exchange)
TAU_EXCHANGE_FN = C.CFUNCTYPE(C.c_int, C.c_void_p, C.c_size_t, C.c_void_p, C.c_void_p)

INDEX_HNSW = 0
INDEX_IVF_PQ = 1
INDEX_DISKANN = 2
SELECT_AUTO = 0
SELECT_MANUAL = 1
SELECT_HYBRID = 2

KMEANS_ELKAN = 0
KMEANS_LLOYD = 1

FLAT_L2 = 0
FLAT_IP = 1


class TrainParams(C.Structure):
    _fields_ = [("nlist", C.c_uint32), ("m", C.c_uint32), ("nbits", C.c_uint32)]


class HnswBuildParams(C.Structure):
    _fields_ = [("M", C.c_uint32), ("ef_construction", C.c_uint32), ("seed", C.c_uint32)]


class VamanaBuildParams(C.Structure):
    _fields_ = [("degree", C.c_uint32), ("L", C.c_uint32), ("alpha", C.c_float)]


class ManagerBuildConfig(C.Structure):
    _fields_ = [("type", C.c_int), ("strategy", C.c_int), ("ivf", TrainParams), ("hnsw", HnswBuildParams),
                ("vamana", VamanaBuildParams)]


class QueryConfig(C.Structure):
    _fields_ = [("k", C.c_uint32), ("epsilon", C.c_float), ("ef_search", C.c_uint32), ("nprobe", C.c_uint32),
                ("l_search", C.c_uint32), ("use_exact_rerank", C.c_int), ("rerank_k", C.c_uint32),
                ("rerank_alpha", C.c_float), ("rerank_cand_ceiling", C.c_uint32), ("use_query_planner", C.c_int),
                ("has_preferred_index", C.c_int), ("preferred_index", C.c_int), ("has_filter", C.c_int),
                ("filter_json", C.c_char_p)]


class IndexStats(C.Structure):
    _fields_ = [("type", C.c_int), ("num_vectors", C.c_size_t), ("memory_usage_bytes", C.c_size_t),
                ("disk_usage_bytes", C.c_size_t), ("build_time_seconds", C.c_float),
                ("avg_query_time_ms", C.c_float), ("measured_recall", C.c_float), ("query_count", C.c_uint64)]


class SearchParams(C.Structure):
    _fields_ = [("k", C.c_uint32), ("nprobe", C.c_uint32)]


class Stats(C.Structure):
    _fields_ = [("n_vectors", C.c_size_t), ("n_lists", C.c_size_t), ("m", C.c_size_t),
                ("memory_bytes", C.c_size_t), ("avg_list_size", C.c_float)]


class TrainParamsEx(C.Structure):
    _fields_ = [("struct_size", C.c_size_t), ("nlist", C.c_uint32), ("m", C.c_uint32),
                ("nbits", C.c_uint32), ("max_iter", C.c_uint32), ("epsilon", C.c_float),
                ("use_opq", C.c_int), ("opq_iter", C.c_uint32), ("opq_sample_n", C.c_size_t),
                ("opq_init_pca", C.c_int), ("seed", C.c_uint32), ("verbose", C.c_int)]


class TrainReport(C.Structure):
    _fields_ = [("opq_kept", C.c_int), ("err_unrot", C.c_double), ("err_opq", C.c_double),
                ("coarse_iterations", C.c_uint32), ("train_time_sec", C.c_float)]


class SearchParamsEx(C.Structure):
    _fields_ = [("struct_size", C.c_size_t), ("k", C.c_uint32), ("nprobe", C.c_uint32),
                ("mode", C.c_uint32), ("cand_k", C.c_uint32), ("use_exact_rerank", C.c_uint32),
                ("rerank_k", C.c_uint32)]


class Timings(C.Structure):
    _fields_ = [("coarse_ms", C.c_float), ("select_ms", C.c_float), ("rotate_ms", C.c_float),
                ("scan_ms", C.c_float), ("merge_ms", C.c_float), ("total_ms", C.c_float),
                ("scanned_entries", C.c_uint64), ("kernel_launches", C.c_uint32),
                ("scan_variant", C.c_uint32), ("coarse_variant", C.c_uint32),
                ("list_kernel_ms", C.c_float), ("list_candidates", C.c_uint64),
                ("list_fallback_queries", C.c_uint32), ("list_threshold_ms", C.c_float),
                ("list_prep_ms", C.c_float), ("list_refine_ms", C.c_float), ("list_fallback_ms", C.c_float),
                ("rerank_ms", C.c_float)]


class KmeansParams(C.Structure):
    _fields_ = [("struct_size", C.c_size_t), ("k", C.c_uint32), ("max_iter", C.c_uint32),
                ("epsilon", C.c_float), ("seed", C.c_uint32), ("algorithm", C.c_uint32)]


class KmeansResult(C.Structure):
    _fields_ = [("iterations", C.c_uint32), ("inertia", C.c_float), ("time_sec", C.c_float)]


class FlatTimings(C.Structure):
    _fields_ = [("total_ms", C.c_float), ("norms_ms", C.c_float), ("sample_ms", C.c_float),
                ("filter_ms", C.c_float), ("refine_ms", C.c_float), ("fallback_ms", C.c_float),
                ("candidates", C.c_uint64), ("overflow_queries", C.c_uint32), ("sample_stride", C.c_uint32),
                ("single_pass", C.c_uint32), ("kernel_launches", C.c_uint32)]


_lib = None
_lock = threading.Lock()


def library_path() -> str:
    return LIB_PATH


def load(path: str = LIB_PATH) -> C.CDLL:
    """Load libvesper_c.so and declare its prototypes (idempotent)."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(path):
            raise RuntimeError(
                f"{path} is missing: build it with `python -m vesper_db_b200.build` "
                "(the engine has no CPU fallback)")
        L = C.CDLL(path)
        vp, st = C.c_void_p, C.c_int
        f32p, u64p, u32p, u8p = (C.POINTER(C.c_float), C.POINTER(C.c_uint64),
                                 C.POINTER(C.c_uint32), C.POINTER(C.c_uint8))
        proto = {
            "vesper_get_last_error": (C.c_char_p, []),
            "vesper_version": (C.c_char_p, []),
            "vesper_ivfpq_create": (st, [C.POINTER(vp)]),
            "vesper_ivfpq_destroy": (st, [vp]),
            "vesper_ivfpq_train": (st, [vp, f32p, C.c_size_t, C.c_size_t, C.POINTER(TrainParams)]),
            "vesper_ivfpq_add": (st, [vp, u64p, f32p, C.c_size_t]),
            "vesper_ivfpq_search": (st, [vp, f32p, C.POINTER(SearchParams), u64p, f32p]),
            "vesper_ivfpq_search_batch": (st, [vp, f32p, C.c_size_t, C.POINTER(SearchParams), u64p, f32p]),
            "vesper_ivfpq_is_trained": (st, [vp, C.POINTER(C.c_int)]),
            "vesper_ivfpq_get_dimension": (st, [vp, C.POINTER(C.c_size_t)]),
            "vesper_ivfpq_get_stats": (st, [vp, C.POINTER(Stats)]),
            "vesper_ivfpq_set_metadata_json": (st, [vp, C.c_char_p]),
            "vesper_ivfpq_get_metadata_json": (st, [vp, C.c_char_p, C.c_size_t, C.POINTER(C.c_size_t)]),
            "vesper_ivfpq_save": (st, [vp, C.c_char_p]),
            "vesper_ivfpq_load": (st, [vp, C.c_char_p]),
            "vesper_ivfpq_train_params_ex_init": (None, [C.POINTER(TrainParamsEx)]),
            "vesper_ivfpq_train_ex": (st, [vp, f32p, C.c_size_t, C.c_size_t, C.POINTER(TrainParamsEx)]),
            "vesper_ivfpq_get_train_report": (st, [vp, C.POINTER(TrainReport)]),
            "vesper_ivfpq_search_batch_ex": (st, [vp, f32p, C.c_size_t, C.POINTER(SearchParamsEx), u64p,
                                                  f32p, u32p]),
            "vesper_ivfpq_search_batch_device": (st, [vp, vp, C.c_size_t, C.POINTER(SearchParamsEx), vp, vp,
                                                      vp]),
            "vesper_ivfpq_get_last_timings": (st, [vp, C.POINTER(Timings)]),
            "vesper_ivfpq_set_model": (st, [vp, C.c_size_t, C.c_uint32, C.c_uint32, C.c_uint32, f32p, f32p,
                                            f32p]),
            "vesper_ivfpq_get_lists": (st, [vp, u64p, u64p, u8p]),
            "vesper_b200_device_count": (C.c_int, []),
            "vesper_ivfpq_train_ex_device": (st, [vp, vp, C.c_size_t, C.c_size_t, C.POINTER(TrainParamsEx)]),
            "vesper_ivfpq_add_device": (st, [vp, vp, vp, C.c_size_t]),
            "vesper_ivfpq_search_batch_device_noalloc": (st, [vp, vp, C.c_size_t, C.POINTER(SearchParamsEx),
                                                              vp, vp, vp]),
            "vesper_kmeans_params_init": (None, [C.POINTER(KmeansParams)]),
            "vesper_kmeans_fit": (st, [f32p, C.c_size_t, C.c_size_t, C.POINTER(KmeansParams), f32p, u32p,
                                       C.POINTER(KmeansResult)]),
            "vesper_kmeans_fit_device": (st, [vp, C.c_size_t, C.c_size_t, C.POINTER(KmeansParams), vp, vp,
                                              C.POINTER(KmeansResult)]),
            "vesper_flat_topk": (st, [C.c_int, f32p, C.c_size_t, f32p, C.c_size_t, C.c_size_t, C.c_uint32,
                                      u32p, f32p]),
            "vesper_flat_topk_device": (st, [C.c_int, vp, C.c_size_t, vp, C.c_size_t, C.c_size_t, C.c_uint32,
                                             vp, vp]),
            "vesper_flat_get_last_timings": (st, [C.POINTER(FlatTimings)]),
            "vesper_ivfpq_probe_device": (st, [vp, vp, C.c_size_t, C.c_uint32, vp, vp]),
            "vesper_ivfpq_search_batch_device_probed": (st, [vp, vp, C.c_size_t, C.POINTER(SearchParamsEx), vp, vp,
                                                             vp, vp, vp]),
            "vesper_ivfpq_set_threshold_exchange": (st, [vp, TAU_EXCHANGE_FN, vp, C.c_uint32, C.c_uint32]),
            "vesper_topk_merge_device": (st, [C.c_uint32, C.c_size_t, C.c_uint32, vp, C.c_size_t, vp, C.c_size_t,
                                              vp, C.c_size_t, vp, vp, vp, vp]),
            "vesper_ivfpq_reconstruct": (st, [vp, C.c_uint64, f32p]),
            "vesper_ivfpq_reconstruct_cluster": (st, [vp, C.c_uint32, u64p, f32p, C.c_size_t,
                                                      C.POINTER(C.c_size_t)]),
            "vesper_ivfpq_get_cluster_assignment": (st, [vp, C.c_uint64, u32p]),
            "vesper_ivfpq_get_cluster_centroid": (st, [vp, C.c_uint32, f32p]),
            "vesper_ivfpq_update_cluster_centroid": (st, [vp, C.c_uint32, f32p]),
            "vesper_ivfpq_reassign_vector": (st, [vp, C.c_uint64, C.c_uint32]),
            "vesper_ivfpq_compact_inverted_list": (st, [vp, C.c_uint32, u32p, C.c_size_t, C.POINTER(C.c_size_t)]),
            "vesper_ivfpq_debug_explain_centroid_rank": (st, [vp, f32p, C.c_uint64, u64p, u32p]),
            "vesper_ivfpq_debug_explain_adc_rank": (st, [vp, f32p, C.c_uint64, u64p, f32p]),
            "vesper_kmeans_shard_create": (st, [C.POINTER(vp)]),
            "vesper_kmeans_shard_destroy": (None, [vp]),
            "vesper_kmeans_shard_assign": (st, [vp, vp, C.c_size_t, C.c_size_t, vp, C.c_uint32, C.c_int, vp, vp]),
            "vesper_kmeans_shard_pp_update": (st, [vp, vp, C.c_size_t, C.c_size_t, vp, vp]),
            "vesper_kmeans_shard_accumulate": (st, [vp, vp, C.c_size_t, C.c_size_t, vp, C.c_uint32, C.c_uint32, vp,
                                                    vp, vp]),
            "vesper_kmeans_shard_finish": (st, [vp, vp, vp, C.c_uint32, C.c_size_t, C.c_uint32, vp]),
            "vesper_kmeans_shard_running_inertia": (st, [vp, vp, C.c_size_t, C.c_size_t, vp, vp,
                                                         C.POINTER(C.c_float)]),
            "vesper_kmeanspp_sampler_create": (st, [C.c_uint32, C.c_size_t, C.POINTER(vp), C.POINTER(C.c_size_t)]),
            "vesper_kmeanspp_sampler_next": (st, [vp, f32p, C.POINTER(C.c_size_t)]),
            "vesper_kmeanspp_sampler_destroy": (None, [vp]),
            "vesper_mgr_create": (st, [C.c_size_t, C.POINTER(vp)]),
            "vesper_mgr_destroy": (st, [vp]),
            "vesper_mgr_build": (st, [vp, f32p, C.c_size_t, C.POINTER(ManagerBuildConfig)]),
            "vesper_mgr_add_batch": (st, [vp, u64p, f32p, C.c_size_t]),
            "vesper_mgr_update": (st, [vp, C.c_uint64, f32p]),
            "vesper_mgr_update_batch": (st, [vp, u64p, f32p, C.c_size_t]),
            "vesper_mgr_remove": (st, [vp, C.c_uint64]),
            "vesper_mgr_remove_batch": (st, [vp, u64p, C.c_size_t]),
            "vesper_mgr_search": (st, [vp, f32p, C.POINTER(QueryConfig), u64p, f32p]),
            "vesper_mgr_search_batch": (st, [vp, f32p, C.c_size_t, C.POINTER(QueryConfig), u64p, f32p]),
            "vesper_mgr_save": (st, [vp, C.c_char_p]),
            "vesper_mgr_load": (st, [vp, C.c_char_p]),
            "vesper_mgr_memory_usage": (st, [vp, C.POINTER(C.c_size_t)]),
            "vesper_mgr_disk_usage": (st, [vp, C.POINTER(C.c_size_t)]),
            "vesper_mgr_set_memory_budget_mb": (st, [vp, C.c_uint32]),
            "vesper_mgr_get_memory_budget_mb": (st, [vp, C.POINTER(C.c_uint32)]),
            "vesper_mgr_get_stats": (st, [vp, C.POINTER(IndexStats), C.POINTER(C.c_size_t), C.POINTER(C.c_size_t)]),
            "vesper_mgr_set_search_mode": (st, [vp, C.c_uint32]),
        }
        for name, (res, args) in proto.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
        return L
