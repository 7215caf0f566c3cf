"""vesper_db_b200: B200-native IVF-PQ/OPQ search, exact flat top-k and k-means training
for Vesper.

The engine is libvesper_c.so (C++ host code + sm_100a CUDA kernels) exporting the
reference's vesper_ivfpq_* C ABI; this package is its Python mirror.
"""
from ._native import SEARCH_EXACT, SEARCH_FAST, library_path, load  # noqa: F401
from .index import IvfPqIndex, TrainReport, VesperError  # noqa: F401
from .flat import flat_topk, flat_topk_device  # noqa: F401
from .kmeans import KmeansResult, kmeans_cluster, kmeans_elkan, kmeans_fit_device  # noqa: F401

__all__ = ["IvfPqIndex", "TrainReport", "VesperError", "SEARCH_FAST", "SEARCH_EXACT", "load",
           "library_path", "KmeansResult", "kmeans_cluster", "kmeans_elkan", "kmeans_fit_device",
           "flat_topk", "flat_topk_device"]
