"""ctypes wrappers for the oracle libraries (test infrastructure only).

``Oracle``     -- liboracle.so, the C++ restatement in vesper_oracle.cpp.
``Reference``  -- _ref/libvesper_ref_nc.so (or libvesper_ref.so), the reference IVF-PQ
                  sources compiled in place plus ref_bridge.cpp.

Only tests/, ``__graft_entry__.smoke()`` and the CPU-baseline leg of bench.py import
this module, and only to check or time the CPU side.  The product package never does.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libvesper_ref.so")
REF_NC_SO = os.path.join(HERE, "_ref", "libvesper_ref_nc.so")

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_u32p = np.ctypeslib.ndpointer(np.uint32, flags="C_CONTIGUOUS")
_u64p = np.ctypeslib.ndpointer(np.uint64, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")
_sz = C.c_size_t
_u32 = C.c_uint32


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def host_threads() -> int:
    """Host CPUs this process may run on (its affinity mask)."""
    try:
        return len(os.sched_getaffinity(0))
    except (AttributeError, OSError):
        return os.cpu_count() or 1


def set_omp_threads(n: int) -> int:
    """Make the reference's OpenMP regions use n threads and return what OpenMP reports.

    torch.distributed.run exports OMP_NUM_THREADS=1 to every rank; libgomp reads the
    variable when it is first loaded, so the variable is set before any library that
    links libgomp is opened, and omp_set_num_threads is called on the loaded copy too."""
    os.environ["OMP_NUM_THREADS"] = str(n)
    try:
        gomp = C.CDLL("libgomp.so.1")
        gomp.omp_set_num_threads(C.c_int(n))
        gomp.omp_get_max_threads.restype = C.c_int
        return int(gomp.omp_get_max_threads())
    except OSError:
        return n


def host_cpu() -> dict:
    """Model name, physical cores and logical CPUs of this host (from /proc/cpuinfo)."""
    model, cores = None, set()
    phys = core = None
    try:
        for line in open("/proc/cpuinfo"):
            key, _, val = line.partition(":")
            key, val = key.strip(), val.strip()
            if key == "model name" and model is None:
                model = val
            elif key == "physical id":
                phys = val
            elif key == "core id":
                core = val
            elif not key and phys is not None and core is not None:
                cores.add((phys, core))
                phys = core = None
        if phys is not None and core is not None:
            cores.add((phys, core))
    except OSError:
        pass
    return {"model": model, "physical_cores": len(cores) or None, "logical_cpus": os.cpu_count(),
            "affinity_cpus": host_threads()}


class Oracle:
    """The restated reference arithmetic (bit-exact with the -ffp-contract=off build)."""

    def __init__(self, path: str = ORACLE_SO):
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} missing: run `make -C oracle oracle`")
        L = self.lib = C.CDLL(path)
        L.orc_l2_sq.restype = C.c_float
        L.orc_l2_sq.argtypes = [_f32p, _f32p, _sz]
        L.orc_inner_product.restype = C.c_float
        L.orc_inner_product.argtypes = [_f32p, _f32p, _sz]
        L.orc_assign.argtypes = [_f32p, _sz, _f32p, _u32, _sz, _u32p, C.c_void_p]
        L.orc_coarse_probe.argtypes = [_f32p, _sz, _f32p, _u32, _sz, _u32, _u32p, _f32p]
        L.orc_rotate.argtypes = [_f32p, _f32p, _sz, _sz, _f32p]
        L.orc_rotate_T.argtypes = [_f32p, _f32p, _sz, _sz, _f32p]
        L.orc_pq_encode.argtypes = [_f32p, _sz, _f32p, _u32, _u32, _sz, _u8p]
        L.orc_pq_decode.argtypes = [_u8p, _sz, _f32p, _u32, _u32, _sz, _f32p]
        L.orc_pq_lut.argtypes = [_f32p, _f32p, _u32, _u32, _sz, _f32p]
        L.orc_adc.restype = C.c_float
        L.orc_adc.argtypes = [_f32p, _u8p, _u32, _u32]
        L.orc_ivfpq_add.argtypes = [_f32p, _sz, _f32p, _u32, _sz, C.c_void_p, _f32p, _u32, _u32,
                                    _u32p, _u8p]
        L.orc_ivfpq_search_batch.argtypes = [_f32p, _sz, _f32p, _u32, _sz, C.c_void_p, _f32p, _u32,
                                             _u32, _u64p, _u64p, _u8p, _u32, _u32, _u64p, _f32p, _u32p]
        L.orc_ivfpq_search_batch_ex.argtypes = [_f32p, _sz, _f32p, _u32, _sz, C.c_void_p, _f32p, _u32,
                                                _u32, _u64p, _u64p, _u8p, _u32, _u32, _u32, C.c_int, _u32,
                                                _u64p, _f32p, _u32p]
        L.orc_flat_topk.argtypes = [C.c_int, _f32p, _sz, _f32p, _u32, _sz, _u32, _u32p, _f32p]
        L.orc_kmeanspp_init.argtypes = [_f32p, _sz, _sz, _u32, _u32, _f32p, _u32p]
        L.orc_lloyd_assign.restype = C.c_float
        L.orc_lloyd_assign.argtypes = [_f32p, _sz, _f32p, _u32, _sz, _u32p]
        L.orc_lloyd_update.argtypes = [_f32p, _sz, _sz, _u32p, _u32, _f32p]
        L.orc_elkan_update_centroid.argtypes = [_f32p, _sz, _u32p, _sz, _u32, _f32p]
        L.orc_kmeans_elkan.restype = C.c_int
        L.orc_kmeans_elkan.argtypes = [_f32p, _sz, _sz, _u32, _u32, C.c_float, _u32, _f32p, _u32p,
                                       C.POINTER(_u32), C.POINTER(C.c_float)]
        L.orc_kmeans_lloyd.restype = C.c_int
        L.orc_kmeans_lloyd.argtypes = L.orc_kmeans_elkan.argtypes
        L.orc_pq_train.restype = C.c_int
        L.orc_pq_train.argtypes = [_f32p, _sz, _sz, _u32, _u32, _f32p]

    # -- primitives
    def l2_sq(self, a, b):
        a, b = _f32(a), _f32(b)
        return float(self.lib.orc_l2_sq(a, b, a.size))

    def inner_product(self, a, b):
        a, b = _f32(a), _f32(b)
        return float(self.lib.orc_inner_product(a, b, a.size))

    def assign(self, x, c):
        x, c = _f32(x), _f32(c)
        out = np.zeros(x.shape[0], np.uint32)
        self.lib.orc_assign(x, x.shape[0], c, c.shape[0], x.shape[1], out, None)
        return out

    def coarse_probe(self, q, c, nprobe):
        q, c = _f32(q), _f32(c)
        npb = min(nprobe, c.shape[0])
        lists = np.zeros((q.shape[0], npb), np.uint32)
        d = np.zeros((q.shape[0], npb), np.float32)
        self.lib.orc_coarse_probe(q, q.shape[0], c, c.shape[0], q.shape[1], nprobe, lists, d)
        return lists, d

    def rotate(self, x, R):
        x, R = _f32(x), _f32(R)
        out = np.zeros_like(x)
        self.lib.orc_rotate(x, R, x.shape[0], x.shape[1], out)
        return out

    def rotate_T(self, x, R):
        x, R = _f32(x), _f32(R)
        out = np.zeros_like(x)
        self.lib.orc_rotate_T(x, R, x.shape[0], x.shape[1], out)
        return out

    def pq_encode(self, x, cb, m):
        """cb: [m*ksub, dsub]."""
        x, cb = _f32(x), _f32(cb)
        ksub = cb.shape[0] // m
        codes = np.zeros((x.shape[0], m), np.uint8)
        self.lib.orc_pq_encode(x, x.shape[0], cb, m, ksub, cb.shape[1], codes)
        return codes

    def pq_decode(self, codes, cb, m):
        codes, cb = np.ascontiguousarray(codes, np.uint8), _f32(cb)
        ksub = cb.shape[0] // m
        out = np.zeros((codes.shape[0], m * cb.shape[1]), np.float32)
        self.lib.orc_pq_decode(codes, codes.shape[0], cb, m, ksub, cb.shape[1], out)
        return out

    def pq_lut(self, r, cb, m):
        r, cb = _f32(r), _f32(cb)
        ksub = cb.shape[0] // m
        lut = np.zeros((m, ksub), np.float32)
        self.lib.orc_pq_lut(r, cb, m, ksub, cb.shape[1], lut)
        return lut

    def adc(self, lut, code):
        lut = _f32(lut)
        code = np.ascontiguousarray(code, np.uint8)
        return float(self.lib.orc_adc(lut, code, lut.shape[0], lut.shape[1]))

    def ivfpq_add(self, x, c, R, cb, m):
        x, c, cb = _f32(x), _f32(c), _f32(cb)
        ksub = cb.shape[0] // m
        assign = np.zeros(x.shape[0], np.uint32)
        codes = np.zeros((x.shape[0], m), np.uint8)
        Rp = None if R is None else _f32(R)
        self.lib.orc_ivfpq_add(x, x.shape[0], c, c.shape[0], x.shape[1],
                               None if Rp is None else Rp.ctypes.data, cb, m, ksub, assign, codes)
        return assign, codes

    def ivfpq_search(self, q, c, R, cb, m, list_offsets, ids, codes, k, nprobe, cand_k=0, rerank=False,
                     rerank_k=0):
        q, c, cb = _f32(q), _f32(c), _f32(cb)
        ksub = cb.shape[0] // m
        nq = q.shape[0]
        out_ids = np.zeros((nq, k), np.uint64)
        out_d = np.zeros((nq, k), np.float32)
        counts = np.zeros(nq, np.uint32)
        Rp = None if R is None else _f32(R)
        self.lib.orc_ivfpq_search_batch_ex(
            q, nq, c, c.shape[0], q.shape[1], None if Rp is None else Rp.ctypes.data, cb, m, ksub,
            np.ascontiguousarray(list_offsets, np.uint64), np.ascontiguousarray(ids, np.uint64),
            np.ascontiguousarray(codes, np.uint8), k, nprobe, cand_k, int(rerank), rerank_k, out_ids, out_d,
            counts)
        return out_ids, out_d, counts

    def manager_search(self, q, c, R, cb, m, list_offsets, ids, codes, k, nprobe, deleted=(), total_deleted=0,
                       use_exact_rerank=False, rerank_k=0, rerank_alpha=2.0, ceiling=2000,
                       filter_by_distance=True):
        """IndexManager::search (src/index/index_manager.cpp:344-585) over an IVF-PQ index
        only: nprobe 0 -> 8; with the exact rerank, cand_k = rerank_k or
        ceil(max(k, alpha * k * log2(1 + nprobe))) capped by the ceiling (:414-436); the
        tombstone filter on (uint32)id -- or, with filter_by_distance, on the truncated
        distance, which is what the reference's TombstoneManager::filter_results reads
        for (id, distance) pairs (tombstone_manager.hpp:150-170); rows left short re-searched
        with k * factor * 1.5, factor = 1 + 1.25 * total_deleted / 100000
        (tombstone_manager.cpp:345-351), at most two nested re-searches; truncated to k.
        Returns per query a list of (id, distance)."""
        import math
        nprobe = nprobe if nprobe > 0 else 8
        dead = set(int(x) & 0xFFFFFFFF for x in deleted)
        factor = np.float32(1.0 + (total_deleted / 100000.0) * 1.25)

        def level(rows, kk, depth):
            # a re-search is a new search() call: the heuristic sees its larger k
            cand_k = 0
            if use_exact_rerank:
                if rerank_k > 0:
                    cand_k = rerank_k
                else:
                    h = max(float(kk), float(np.float32(rerank_alpha)) * float(kk) * math.log2(1.0 + nprobe))
                    cand_k = int(math.ceil(h))
                    if ceiling > 0:
                        cand_k = min(cand_k, ceiling)
            rr_k = rerank_k if rerank_k > 0 else cand_k
            rid, rd, rcnt = self.ivfpq_search(q[rows], c, R, cb, m, list_offsets, ids, codes, kk, nprobe,
                                              cand_k=cand_k, rerank=use_exact_rerank, rerank_k=rr_k)
            res = []
            for i in range(len(rows)):
                keep = []
                for j in range(int(rcnt[i])):
                    key = int(np.float32(rd[i, j])) & 0xFFFFFFFF if filter_by_distance else int(rid[i, j]) & 0xFFFFFFFF
                    if key not in dead:
                        keep.append((int(rid[i, j]), float(rd[i, j])))
                res.append(keep)
            short = [i for i in range(len(rows)) if len(res[i]) < kk]
            if short and factor > np.float32(1.0) and depth < 2:
                k2 = int(np.float32(np.float32(kk) * factor) * np.float32(1.5))
                again = level([rows[i] for i in short], k2, depth + 1)
                for j, i in enumerate(short):
                    if len(again[j]) >= kk:
                        res[i] = again[j]
            return [r[:kk] for r in res]

        return level(list(range(q.shape[0])), k, 0)

    # ---- the rest of IvfPqIndex's API (src/index/ivf_pq.cpp:4997-5321, 5392-5541) on a
    # CSR index (list_offsets, ids, codes in list order), restated with the primitives above.
    @staticmethod
    def find_entry(ids, vid):
        """The first entry in list order holding vid (the reference's linear search), or None."""
        hit = np.flatnonzero(np.asarray(ids, np.uint64) == np.uint64(vid))
        return int(hit[0]) if hit.size else None

    @staticmethod
    def list_of(list_offsets, e):
        return int(np.searchsorted(np.asarray(list_offsets, np.uint64), np.uint64(e), side="right") - 1)

    def reconstruct_entries(self, centroids, R, cb, m, lists, codes):
        """centroid + apply_rotation_T(decode(code)) (reconstruct, ivf_pq.cpp:5064-5117)."""
        res = self.pq_decode(codes, cb, m)
        if R is not None:
            res = self.rotate_T(res, R)
        return (_f32(centroids)[np.asarray(lists)] + res).astype(np.float32)

    def reassign(self, centroids, R, cb, m, list_offsets, ids, codes, vid, new_cluster):
        """reassign_vector (ivf_pq.cpp:5226-5321): remove the entry, re-encode the
        reconstructed vector against the new centroid, append it to the new list."""
        offs = np.asarray(list_offsets, np.uint64).astype(np.int64)
        ids = np.asarray(ids, np.uint64)
        codes = np.ascontiguousarray(codes, np.uint8)
        e = self.find_entry(ids, vid)
        lo = self.list_of(offs, e)
        vec = self.reconstruct_entries(centroids, R, cb, m, [lo], codes[e:e + 1])
        r = (vec - _f32(centroids)[new_cluster:new_cluster + 1]).astype(np.float32)
        if R is not None:
            r = self.rotate(r, R)
        code = self.pq_encode(r, cb, m)
        keep = np.ones(ids.shape[0], bool)
        keep[e] = False
        nl = offs.shape[0] - 1
        new_ids, new_codes, new_offs = [], [], [0]
        for l in range(nl):
            sl = slice(offs[l], offs[l + 1])
            li, lc = ids[sl][keep[sl]], codes[sl][keep[sl]]
            if l == new_cluster:
                li = np.concatenate([li, np.array([vid], np.uint64)])
                lc = np.concatenate([lc, code])
            new_ids.append(li)
            new_codes.append(lc)
            new_offs.append(new_offs[-1] + li.shape[0])
        return (np.array(new_offs, np.uint64), np.concatenate(new_ids),
                np.concatenate(new_codes).reshape(-1, m))

    def centroid_rank(self, q, centroids, cluster):
        """debug_explain_centroid_rank: 1 + #centroids strictly closer than the target's."""
        d = np.array([self.l2_sq(q, c) for c in _f32(centroids)], np.float32)
        return int(np.sum(d < d[cluster])) + 1

    def adc_all(self, q, centroids, R, cb, m, list_offsets, codes):
        """The exact ADC distance of q to every entry (its list's table, reference order)."""
        offs = np.asarray(list_offsets, np.uint64).astype(np.int64)
        codes = np.ascontiguousarray(codes, np.uint8)
        out = np.zeros(codes.shape[0], np.float32)
        for l in range(offs.shape[0] - 1):
            if offs[l + 1] == offs[l]:
                continue
            r = (_f32(q)[None, :] - _f32(centroids)[l:l + 1]).astype(np.float32)
            if R is not None:
                r = self.rotate(r, R)
            lut = self.pq_lut(r[0], cb, m)
            for e in range(offs[l], offs[l + 1]):
                out[e] = self.adc(lut, codes[e])
        return out

    def flat_topk(self, op, q, base, k):
        q, base = _f32(q), _f32(base)
        idx = np.zeros((q.shape[0], k), np.uint32)
        sc = np.zeros((q.shape[0], k), np.float32)
        self.lib.orc_flat_topk(op, q, q.shape[0], base, base.shape[0], q.shape[1], k, idx, sc)
        return idx, sc

    def kmeanspp_init(self, x, k, seed):
        x = _f32(x)
        c = np.zeros((k, x.shape[1]), np.float32)
        idx = np.zeros(k, np.uint32)
        self.lib.orc_kmeanspp_init(x, x.shape[0], x.shape[1], k, seed, c, idx)
        return c, idx

    def lloyd_assign(self, x, c):
        x, c = _f32(x), _f32(c)
        out = np.zeros(x.shape[0], np.uint32)
        inertia = self.lib.orc_lloyd_assign(x, x.shape[0], c, c.shape[0], x.shape[1], out)
        return out, float(inertia)

    def lloyd_update(self, x, assign, c):
        x = _f32(x)
        c = _f32(c).copy()
        self.lib.orc_lloyd_update(x, x.shape[0], x.shape[1], np.ascontiguousarray(assign, np.uint32),
                                  c.shape[0], c)
        return c

    def elkan_update(self, x, assign, c):
        x = _f32(x)
        c = _f32(c).copy()
        self.lib.orc_elkan_update_centroid(x, x.shape[1], np.ascontiguousarray(assign, np.uint32),
                                           x.shape[0], c.shape[0], c)
        return c

    def kmeans_elkan(self, x, k, max_iter=25, eps=1e-4, seed=42):
        x = _f32(x)
        c = np.zeros((k, x.shape[1]), np.float32)
        a = np.zeros(x.shape[0], np.uint32)
        it = _u32(0)
        inertia = C.c_float(0)
        rc = self.lib.orc_kmeans_elkan(x, x.shape[0], x.shape[1], k, max_iter, eps, seed, c, a,
                                       C.byref(it), C.byref(inertia))
        if rc != 0:
            raise ValueError("kmeans_elkan: n < k")
        return c, a, it.value, inertia.value

    def kmeans_lloyd(self, x, k, max_iter=25, eps=1e-4, seed=42):
        x = _f32(x)
        c = np.zeros((k, x.shape[1]), np.float32)
        a = np.zeros(x.shape[0], np.uint32)
        it = _u32(0)
        inertia = C.c_float(0)
        rc = self.lib.orc_kmeans_lloyd(x, x.shape[0], x.shape[1], k, max_iter, eps, seed, c, a,
                                       C.byref(it), C.byref(inertia))
        if rc != 0:
            raise ValueError("kmeans_lloyd: n < k or k == 0")
        return c, a, it.value, inertia.value

    def pq_train(self, x, m, nbits):
        x = _f32(x)
        dsub = x.shape[1] // m
        cb = np.zeros(((1 << nbits) * m, dsub), np.float32)
        rc = self.lib.orc_pq_train(x, x.shape[0], x.shape[1], m, nbits, cb)
        if rc != 0:
            raise ValueError("pq_train: dim % m != 0")
        return cb


class Reference:
    """The reference implementation itself, compiled from its sources (oracle/Makefile)."""

    def __init__(self, path: str = REF_NC_SO):
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} missing: run `make -C oracle ref` where the reference is mounted")
        L = self.lib = C.CDLL(path)
        L.rb_last_error.restype = C.c_char_p
        L.rb_l2_sq.restype = C.c_float
        L.rb_l2_sq.argtypes = [_f32p, _f32p, _sz]
        L.rb_inner_product.restype = C.c_float
        L.rb_inner_product.argtypes = [_f32p, _f32p, _sz]
        L.rb_ivfpq_create.restype = C.c_void_p
        L.rb_ivfpq_destroy.argtypes = [C.c_void_p]
        L.rb_ivfpq_train.restype = C.c_int
        L.rb_ivfpq_train.argtypes = [C.c_void_p, _f32p, _sz, _sz, _u32, _u32, _u32, C.c_int, C.c_int,
                                     _u32, C.c_float, _u32, _sz, _u32]
        L.rb_ivfpq_add.restype = C.c_int
        L.rb_ivfpq_add.argtypes = [C.c_void_p, _u64p, _f32p, _sz]
        L.rb_ivfpq_search_batch.restype = C.c_int
        L.rb_ivfpq_search_batch.argtypes = [C.c_void_p, _f32p, _sz, _u32, _u32, _u64p, _f32p, _u32p]
        for name, args in {
                "rb_ivfpq_reconstruct": [C.c_void_p, C.c_uint64, _f32p],
                "rb_ivfpq_reconstruct_cluster": [C.c_void_p, _u32, _u64p, _f32p, _sz, C.POINTER(C.c_size_t)],
                "rb_ivfpq_get_cluster_assignment": [C.c_void_p, C.c_uint64, C.POINTER(C.c_uint32)],
                "rb_ivfpq_update_cluster_centroid": [C.c_void_p, _u32, _f32p],
                "rb_ivfpq_reassign_vector": [C.c_void_p, C.c_uint64, _u32],
                "rb_ivfpq_debug_centroid_rank": [C.c_void_p, _f32p, C.c_uint64, C.POINTER(C.c_uint64),
                                                 C.POINTER(C.c_uint32)],
                "rb_ivfpq_debug_adc_rank": [C.c_void_p, _f32p, C.c_uint64, C.POINTER(C.c_uint64),
                                            C.POINTER(C.c_float)]}.items():
            getattr(L, name).restype = C.c_int
            getattr(L, name).argtypes = args
        L.rb_flat_buffer_create.restype = C.c_void_p
        L.rb_flat_buffer_create.argtypes = [_f32p, _u32, _sz]
        L.rb_flat_buffer_destroy.argtypes = [C.c_void_p]
        L.rb_flat_topk_buffer.argtypes = [C.c_int, _f32p, _sz, C.c_void_p, _u32, _u32p, _f32p]
        L.rb_ivfpq_search_batch_ex.restype = C.c_int
        L.rb_ivfpq_search_batch_ex.argtypes = [C.c_void_p, _f32p, _sz, _u32, _u32, _u32, C.c_int, _u32, _u64p,
                                               _f32p, _u32p]
        L.rb_ivfpq_save.restype = C.c_int
        L.rb_ivfpq_save.argtypes = [C.c_void_p, C.c_char_p]
        L.rb_ivfpq_load.restype = C.c_int
        L.rb_ivfpq_load.argtypes = [C.c_void_p, C.c_char_p]
        L.rb_ivfpq_set_metadata_json.restype = None
        L.rb_ivfpq_set_metadata_json.argtypes = [C.c_void_p, C.c_char_p]
        L.rb_ivfpq_get_metadata_json.restype = C.c_size_t
        L.rb_ivfpq_get_metadata_json.argtypes = [C.c_void_p, C.c_char_p, C.c_size_t]
        L.rb_kmeanspp_init.argtypes = [_f32p, _sz, _sz, _u32, _u32, _f32p]
        for fn in ("rb_kmeans_elkan", "rb_kmeans_lloyd"):
            getattr(L, fn).restype = C.c_int
            getattr(L, fn).argtypes = [_f32p, _sz, _sz, _u32, _u32, C.c_float, _u32, _f32p, _u32p,
                                       C.POINTER(_u32), C.POINTER(C.c_float)]
        L.rb_kmeans_assign.restype = C.c_float
        L.rb_kmeans_assign.argtypes = [_f32p, _sz, _f32p, _u32, _sz, _u32p]
        L.rb_kmeans_update.argtypes = [_f32p, _sz, _sz, _u32p, _u32, _f32p]
        L.rb_pq_create.restype = C.c_void_p
        L.rb_pq_create.argtypes = [_u32, _u32]
        L.rb_pq_destroy.argtypes = [C.c_void_p]
        L.rb_pq_train.restype = C.c_int
        L.rb_pq_train.argtypes = [C.c_void_p, _f32p, _sz, _sz]
        L.rb_pq_import.argtypes = [C.c_void_p, _sz, _f32p, _sz]
        L.rb_pq_export.argtypes = [C.c_void_p, _f32p]
        L.rb_pq_encode.argtypes = [C.c_void_p, _f32p, _sz, _u8p]
        L.rb_pq_lut.argtypes = [C.c_void_p, _f32p, _f32p]
        L.rb_pq_adc.argtypes = [C.c_void_p, _f32p, _u8p, _sz, _f32p]
        L.rb_flat_topk.argtypes = [C.c_int, _f32p, _sz, _f32p, _u32, _sz, _u32, _u32p, _f32p]

    def error(self):
        return self.lib.rb_last_error().decode()

    def l2_sq(self, a, b):
        a, b = _f32(a), _f32(b)
        return float(self.lib.rb_l2_sq(a, b, a.size))

    def inner_product(self, a, b):
        a, b = _f32(a), _f32(b)
        return float(self.lib.rb_inner_product(a, b, a.size))

    def kmeanspp_init(self, x, k, seed):
        x = _f32(x)
        c = np.zeros((k, x.shape[1]), np.float32)
        self.lib.rb_kmeanspp_init(x, x.shape[0], x.shape[1], k, seed, c)
        return c

    def _kmeans(self, fn, x, k, max_iter, eps, seed):
        x = _f32(x)
        c = np.zeros((k, x.shape[1]), np.float32)
        a = np.zeros(x.shape[0], np.uint32)
        it = _u32(0)
        inertia = C.c_float(0)
        rc = fn(x, x.shape[0], x.shape[1], k, max_iter, eps, seed, c, a, C.byref(it), C.byref(inertia))
        if rc != 0:
            raise ValueError(self.error())
        return c, a, it.value, inertia.value

    def kmeans_elkan(self, x, k, max_iter=25, eps=1e-4, seed=42):
        return self._kmeans(self.lib.rb_kmeans_elkan, x, k, max_iter, eps, seed)

    def kmeans_lloyd(self, x, k, max_iter=25, eps=1e-4, seed=42):
        return self._kmeans(self.lib.rb_kmeans_lloyd, x, k, max_iter, eps, seed)

    def kmeans_assign(self, x, c):
        x, c = _f32(x), _f32(c)
        out = np.zeros(x.shape[0], np.uint32)
        inertia = self.lib.rb_kmeans_assign(x, x.shape[0], c, c.shape[0], x.shape[1], out)
        return out, float(inertia)

    def kmeans_update(self, x, assign, c):
        x = _f32(x)
        c = _f32(c).copy()
        self.lib.rb_kmeans_update(x, x.shape[0], x.shape[1], np.ascontiguousarray(assign, np.uint32),
                                  c.shape[0], c)
        return c

    def flat_topk(self, op, q, base, k):
        q, base = _f32(q), _f32(base)
        idx = np.zeros((q.shape[0], k), np.uint32)
        sc = np.zeros((q.shape[0], k), np.float32)
        self.lib.rb_flat_topk(op, q, q.shape[0], base, base.shape[0], q.shape[1], k, idx, sc)
        return idx, sc

    def flat_buffer(self, base):
        """The base copied once into the reference's AlignedCentroidBuffer; returns an
        object whose topk(op, q, k) runs find_nearest_centroids_batch_fused on it."""
        return RefFlatBuffer(self, base)

    def pq(self, m, nbits):
        return RefPq(self, m, nbits)

    def ivfpq(self):
        return RefIvfPq(self)


class RefFlatBuffer:
    def __init__(self, ref: Reference, base):
        base = _f32(base)
        self.ref, self.nb = ref, base.shape[0]
        self.h = ref.lib.rb_flat_buffer_create(base, base.shape[0], base.shape[1])

    def __del__(self):
        if getattr(self, "h", None):
            self.ref.lib.rb_flat_buffer_destroy(self.h)
            self.h = None

    def topk(self, op, q, k):
        q = _f32(q)
        idx = np.zeros((q.shape[0], k), np.uint32)
        sc = np.zeros((q.shape[0], k), np.float32)
        self.ref.lib.rb_flat_topk_buffer(op, q, q.shape[0], self.h, k, idx, sc)
        return idx, sc


class RefPq:
    def __init__(self, ref: Reference, m: int, nbits: int):
        self.ref, self.m, self.ksub = ref, m, 1 << nbits
        self.h = ref.lib.rb_pq_create(m, nbits)
        self.dsub = 0

    def __del__(self):
        if getattr(self, "h", None):
            self.ref.lib.rb_pq_destroy(self.h)
            self.h = None

    def train(self, x):
        x = _f32(x)
        self.dsub = x.shape[1] // self.m
        if self.ref.lib.rb_pq_train(self.h, x, x.shape[0], x.shape[1]) != 0:
            raise ValueError(self.ref.error())

    def import_codebooks(self, cb):
        cb = _f32(cb)
        self.dsub = cb.shape[1]
        self.ref.lib.rb_pq_import(self.h, cb.shape[1], cb, cb.size)

    def codebooks(self):
        out = np.zeros((self.m * self.ksub, self.dsub), np.float32)
        self.ref.lib.rb_pq_export(self.h, out)
        return out

    def encode(self, x):
        x = _f32(x)
        codes = np.zeros((x.shape[0], self.m), np.uint8)
        self.ref.lib.rb_pq_encode(self.h, x, x.shape[0], codes)
        return codes

    def lut(self, q):
        out = np.zeros((self.m, self.ksub), np.float32)
        self.ref.lib.rb_pq_lut(self.h, _f32(q), out)
        return out

    def adc(self, q, codes):
        codes = np.ascontiguousarray(codes, np.uint8)
        out = np.zeros(codes.shape[0], np.float32)
        self.ref.lib.rb_pq_adc(self.h, _f32(q), codes, codes.shape[0], out)
        return out


class RefIvfPq:
    def __init__(self, ref: Reference):
        self.ref = ref
        self.h = ref.lib.rb_ivfpq_create()

    def __del__(self):
        if getattr(self, "h", None):
            self.ref.lib.rb_ivfpq_destroy(self.h)
            self.h = None

    def train(self, x, nlist, m, nbits=8, use_opq=False, brute_assign=True, max_iter=25,
              epsilon=1e-4, seed=42, opq_sample_n=20000, opq_iter=10):
        x = _f32(x)
        rc = self.ref.lib.rb_ivfpq_train(self.h, x, x.shape[1], x.shape[0], nlist, m, nbits,
                                         int(use_opq), int(brute_assign), max_iter, epsilon, seed,
                                         opq_sample_n, opq_iter)
        if rc != 0:
            raise ValueError(self.ref.error())

    def add(self, ids, x):
        x = _f32(x)
        rc = self.ref.lib.rb_ivfpq_add(self.h, np.ascontiguousarray(ids, np.uint64), x, x.shape[0])
        if rc != 0:
            raise ValueError(self.ref.error())

    def search(self, q, k, nprobe, cand_k=0, rerank=False, rerank_k=0):
        q = _f32(q)
        nq = q.shape[0]
        ids = np.zeros((nq, k), np.uint64)
        d = np.zeros((nq, k), np.float32)
        counts = np.zeros(nq, np.uint32)
        if cand_k or rerank or rerank_k:
            rc = self.ref.lib.rb_ivfpq_search_batch_ex(self.h, q, nq, k, nprobe, cand_k, int(rerank), rerank_k,
                                                       ids, d, counts)
        else:
            rc = self.ref.lib.rb_ivfpq_search_batch(self.h, q, nq, k, nprobe, ids, d, counts)
        if rc != 0:
            raise ValueError(self.ref.error())
        return ids, d, counts

    def reconstruct(self, vid, dim):
        out = np.zeros(dim, np.float32)
        rc = self.ref.lib.rb_ivfpq_reconstruct(self.h, vid, out)
        return rc, out

    def reconstruct_cluster(self, cluster, dim, cap=1 << 20):
        ids = np.zeros(cap, np.uint64)
        vec = np.zeros(cap * dim, np.float32)
        n = C.c_size_t(0)
        rc = self.ref.lib.rb_ivfpq_reconstruct_cluster(self.h, cluster, ids, vec, cap, C.byref(n))
        return rc, ids[:n.value], vec[:n.value * dim].reshape(n.value, dim)

    def get_cluster_assignment(self, vid):
        out = C.c_uint32(0)
        rc = self.ref.lib.rb_ivfpq_get_cluster_assignment(self.h, vid, C.byref(out))
        return rc, out.value

    def update_cluster_centroid(self, cluster, c):
        return self.ref.lib.rb_ivfpq_update_cluster_centroid(self.h, cluster, _f32(c))

    def reassign_vector(self, vid, cluster):
        return self.ref.lib.rb_ivfpq_reassign_vector(self.h, vid, cluster)

    def debug_centroid_rank(self, q, vid):
        rank, cl = C.c_uint64(0), C.c_uint32(0)
        rc = self.ref.lib.rb_ivfpq_debug_centroid_rank(self.h, _f32(q), vid, C.byref(rank), C.byref(cl))
        return rc, rank.value, cl.value

    def debug_adc_rank(self, q, vid):
        rank, d = C.c_uint64(0), C.c_float(0)
        rc = self.ref.lib.rb_ivfpq_debug_adc_rank(self.h, _f32(q), vid, C.byref(rank), C.byref(d))
        return rc, rank.value, d.value

    def save(self, directory):
        if self.ref.lib.rb_ivfpq_save(self.h, directory.encode()) != 0:
            raise IOError(self.ref.error())

    def load(self, directory):
        if self.ref.lib.rb_ivfpq_load(self.h, directory.encode()) != 0:
            raise IOError(self.ref.error())

    def set_metadata_json(self, js: str):
        self.ref.lib.rb_ivfpq_set_metadata_json(self.h, js.encode())

    def get_metadata_json(self) -> str:
        n = self.ref.lib.rb_ivfpq_get_metadata_json(self.h, None, 0)
        buf = C.create_string_buffer(n + 1)
        self.ref.lib.rb_ivfpq_get_metadata_json(self.h, buf, n + 1)
        return buf.value.decode()


def _fnv1a64(data: bytes) -> int:
    h = 1469598103934665603
    for b in data:
        h = ((h ^ b) * 1099511628211) & 0xFFFFFFFFFFFFFFFF
    return h


def _parse_lists(raw: bytes, off: int, m: int):
    """[lists_count u32][per list: size u64, size x (id u64, m code bytes)] -> CSR."""
    lists_count = int(np.frombuffer(raw, np.uint32, 1, off)[0]); off += 4
    offs = np.zeros(lists_count + 1, np.uint64)
    ids, codes = [], []
    for li in range(lists_count):
        sz = int(np.frombuffer(raw, np.uint64, 1, off)[0]); off += 8
        rec = np.frombuffer(raw, np.uint8, sz * (8 + m), off).reshape(sz, 8 + m); off += sz * (8 + m)
        ids.append(rec[:, :8].copy().view(np.uint64).reshape(-1))
        codes.append(rec[:, 8:].copy())
        offs[li + 1] = offs[li] + sz
    return off, offs, (np.concatenate(ids) if ids else np.zeros(0, np.uint64)), \
        (np.concatenate(codes) if codes else np.zeros((0, m), np.uint8))


def read_ivfpq(path: str) -> dict:
    """Parse an ``ivfpq.bin`` file as IvfPqIndex::save writes it (src/index/ivf_pq.cpp:
    4270-4491), v1.0 monolithic or v1.1 sectioned (uncompressed sections), into arrays:
    centroids, codebooks [m*ksub, dsub], rotation or None, metadata (str), and the
    inverted lists as CSR (list_offsets, ids, codes) in list order, entries in file
    order.  Verifies the FNV-1a-64 trailer and, for v1.1, every section checksum;
    `sections` lists the v1.1 section types in file order."""
    raw = open(path, "rb").read()
    magic = raw[:8]
    if magic not in (b"IVFPQv10", b"IVFPQv11"):
        raise ValueError("not an IVF-PQ file")
    v11 = magic == b"IVFPQv11"
    if raw[-12:-8] != b"CHKS" or int.from_bytes(raw[-8:], "little") != _fnv1a64(raw[:-12]):
        raise ValueError("checksum mismatch")
    off = 8
    ver_major, ver_minor = np.frombuffer(raw, np.uint16, 2, off); off += 4
    flags, dim, nlist, m, nbits, dsub = np.frombuffer(raw, np.uint32, 6, off); off += 24
    nvec = int(np.frombuffer(raw, np.uint64, 1, off)[0]); off += 8
    code_size = int(np.frombuffer(raw, np.uint32, 1, off)[0]); off += 4
    off += 8  # build timestamp
    meta_len = int(np.frombuffer(raw, np.uint32, 1, off)[0]); off += 4
    meta = raw[off:off + meta_len].decode(); off += meta_len
    dim, nlist, m, nbits, dsub = int(dim), int(nlist), int(m), int(nbits), int(dsub)
    ksub = 1 << nbits
    R = None
    sections = []
    if v11:
        end = len(raw) - 12
        payloads = {}
        while off + 28 <= end:
            typ = int(np.frombuffer(raw, np.uint32, 1, off)[0])
            unc, comp, shash = (int(v) for v in np.frombuffer(raw, np.uint64, 3, off + 4))
            off += 28
            if comp != unc:
                raise ValueError("compressed section")
            data = raw[off:off + comp]; off += comp
            if _fnv1a64(data) != shash:
                raise ValueError("section checksum mismatch")
            sections.append(typ)
            payloads[typ] = data
        cent = np.frombuffer(payloads[1], np.float32).reshape(nlist, dim).copy()
        cb = np.frombuffer(payloads[2], np.float32).reshape(m * ksub, dsub).copy()
        if 4 in payloads:
            R = np.frombuffer(payloads[4], np.float32).reshape(dim, dim).copy()
        if 5 in payloads:
            meta = payloads[5].decode()
        _, offs, ids, codes = _parse_lists(payloads[3], 0, m)
    else:
        cent = np.frombuffer(raw, np.float32, nlist * dim, off).reshape(nlist, dim).copy(); off += nlist * dim * 4
        cb = np.frombuffer(raw, np.float32, m * ksub * dsub, off).reshape(m * ksub, dsub).copy(); off += cb.nbytes
        if flags & 1:
            R = np.frombuffer(raw, np.float32, dim * dim, off).reshape(dim, dim).copy(); off += R.nbytes
        _, offs, ids, codes = _parse_lists(raw, off, m)
    return dict(version=(int(ver_major), int(ver_minor)), dim=dim, nlist=nlist, m=m, nbits=nbits, dsub=dsub,
                nvec=nvec, flags=int(flags), code_size=code_size, centroids=cent, codebooks=cb, rotation=R,
                metadata=meta, sections=sections, list_offsets=offs, ids=ids, codes=codes)


def read_ivfpq_v10(path: str) -> dict:
    """read_ivfpq restricted to v1.0 files."""
    if open(path, "rb").read(8) != b"IVFPQv10":
        raise ValueError("not a v1.0 IVF-PQ file")
    return read_ivfpq(path)
