"""Python mirror of the reference's k-means entry points over the B200 C ABI.

`kmeans_cluster` follows include/vesper/index/kmeans.hpp:49-62 (one run of Lloyd from
k-means++; `KmeansResult` fields centroids / assignments / cluster_sizes / inertia /
iterations / time_sec) and `kmeans_elkan` follows KmeansElkan::cluster
(src/index/kmeans_elkan.cpp:293-430).  Both call vesper_kmeans_fit (host arrays) or
vesper_kmeans_fit_device (device pointers) in libvesper_c.so.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np

from . import _native as N
from .index import VesperError, _check, _f32, _ptr


@dataclass
class KmeansResult:
    centroids: np.ndarray        # [k, dim] float32
    assignments: np.ndarray      # [n] uint32
    cluster_sizes: np.ndarray    # [k] uint32
    inertia: float
    iterations: int
    time_sec: float


def _params(k, max_iter, epsilon, seed, algorithm):
    lib = N.load()
    p = N.KmeansParams()
    lib.vesper_kmeans_params_init(C.byref(p))
    p.k, p.max_iter, p.epsilon, p.seed, p.algorithm = k, max_iter, epsilon, seed, algorithm
    return lib, p


def _fit(data, k, max_iter, epsilon, seed, algorithm) -> KmeansResult:
    x = _f32(data)
    if x.ndim != 2:
        raise VesperError(N.VESPER_ERROR_INVALID_PARAM, "data must be [n, dim]")
    n, dim = x.shape
    lib, p = _params(k, max_iter, epsilon, seed, algorithm)
    c = np.zeros((max(k, 1), dim), np.float32)
    a = np.zeros(n, np.uint32)
    r = N.KmeansResult()
    _check(lib, lib.vesper_kmeans_fit(_ptr(x, C.c_float), n, dim, C.byref(p), _ptr(c, C.c_float),
                                      _ptr(a, C.c_uint32), C.byref(r)))
    sizes = np.bincount(a, minlength=k).astype(np.uint32)
    return KmeansResult(c, a, sizes, float(r.inertia), int(r.iterations), float(r.time_sec))


def kmeans_cluster(data, k: int, max_iter: int = 25, epsilon: float = 1e-4, seed: int = 42) -> KmeansResult:
    """Lloyd k-means (src/index/kmeans.cpp:137-252, n_redo = 1) on the GPU."""
    return _fit(data, k, max_iter, epsilon, seed, N.KMEANS_LLOYD)


def kmeans_elkan(data, k: int, max_iter: int = 25, epsilon: float = 1e-4, seed: int = 42) -> KmeansResult:
    """KmeansElkan::cluster semantics (src/index/kmeans_elkan.cpp:293-430) on the GPU."""
    return _fit(data, k, max_iter, epsilon, seed, N.KMEANS_ELKAN)


def kmeans_fit_device(x_ptr: int, n: int, dim: int, k: int, c_ptr: int, a_ptr: int = 0, max_iter: int = 25,
                      epsilon: float = 1e-4, seed: int = 42, algorithm: int = N.KMEANS_ELKAN) -> tuple[int, float]:
    """Device-resident fit: x [n, dim] f32, centroids [k, dim] f32 and assignments [n] u32
    are device addresses (e.g. torch data_ptr()).  Returns (iterations, inertia)."""
    lib, p = _params(k, max_iter, epsilon, seed, algorithm)
    r = N.KmeansResult()
    _check(lib, lib.vesper_kmeans_fit_device(C.c_void_p(x_ptr), n, dim, C.byref(p), C.c_void_p(c_ptr),
                                             C.c_void_p(a_ptr) if a_ptr else None, C.byref(r)))
    return int(r.iterations), float(r.inertia)
