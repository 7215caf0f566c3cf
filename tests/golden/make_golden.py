"""Generate the golden fixtures in tests/golden/ from the reference implementation.

Run where the reference sources are mounted and oracle/_ref is built
(`make -C oracle`):

    python tests/golden/make_golden.py <reference source root>   # or VESPER_REFERENCE_DIR set

Outputs (all small, committed):
  pq_lut_small.json     algorithms/fixtures/pq/pq_lut_small.json with its arithmetic
                        expressions evaluated (the original is not valid JSON)
  l2_ip_small.json      algorithms/fixtures/distance_kernels/l2_ip_small.json
  ivfpq_<case>/ivfpq.bin   indexes trained and filled by the reference IvfPqIndex
                           (brute-force coarse assigner), saved by its own save()
  ivfpq_<case>.npz      the base vectors and queries used, and the reference's
                        search results for several (k, nprobe)
  kmeans_small.npz      reference k-means++ / Elkan / Lloyd / PQ-train outputs
  ivfpq_<case>_rerank.npz  the reference's searches with the exact rerank on the saved
                           indexes (`--rerank-only` regenerates just these)
  ivfpq_<case>_api.npz     reconstruct / reconstruct_cluster / get_cluster_assignment /
                           debug rank explanations, and update_cluster_centroid +
                           reassign_vector with the index they leave (ivfpq_<case>_api/)
                           (`--api-only` regenerates just these)
  ivfpq_<case>_v11/ivfpq.bin  the golden index re-saved by the reference in the v1.1
                              sectioned layout (VESPER_IVFPQ_SAVE_V11=1), one case with
                              JSON metadata; ivfpq_v11.json records the metadata and the
                              reference's answers to invalid metadata (`--v11-only`)
"""
from __future__ import annotations

import json
import os
import re
import shutil
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "..", "..", "oracle"))
from oracle_lib import Reference  # noqa: E402

# (case name, dim, nlist, m, use_opq, n_base, n_train, mixture centres, sigma)
CASES = [
    ("plain_d32_m8", 32, 16, 8, False, 2000, 1500, 40, 0.1),    # dsub = 4 (all scalar tail)
    ("plain_d64_m8", 64, 24, 8, False, 2000, 1500, 50, 0.1),    # dsub = 8 (one FMA lane step)
    ("opq_d32_m4", 32, 16, 4, True, 2000, 1500, 40, 0.2),       # OPQ kept/dropped by the reference
    ("odd_d20_m5", 20, 8, 5, False, 800, 600, 20, 0.1),         # dim % 8 != 0 coarse tail
    ("plain_d64_n128", 64, 128, 16, False, 6000, 4000, 300, 0.1),  # nlist >= 64: tensor-core coarse path
]
SEARCHES = [(10, 4), (10, 16), (100, 8), (5, 1), (3, 64)]


def mixture(n, d, ncent, sigma, seed):
    g = np.random.default_rng(seed)
    cent = g.uniform(-1, 1, (ncent, d)).astype(np.float32)
    lab = g.integers(0, ncent, n)
    return (cent[lab] + sigma * g.standard_normal((n, d))).astype(np.float32)


def convert_fixtures(ref_root):
    src = os.path.join(ref_root, "algorithms", "fixtures", "pq", "pq_lut_small.json")
    text = open(src).read()
    # evaluate "a + b" literal expressions so the file parses as JSON
    text = re.sub(r"(-?\d+\.\d+)\s*\+\s*(-?\d+\.\d+)", lambda mt: repr(float(mt.group(1)) + float(mt.group(2))), text)
    json.dump(json.loads(text), open(os.path.join(HERE, "pq_lut_small.json"), "w"), indent=1)
    src = os.path.join(ref_root, "algorithms", "fixtures", "distance_kernels", "l2_ip_small.json")
    json.dump(json.load(open(src)), open(os.path.join(HERE, "l2_ip_small.json"), "w"), indent=1)


def make_ivfpq(ref: Reference):
    for (name, d, nlist, m, opq, nb, nt, nc, sigma) in CASES:
        x = mixture(nb, d, nc, sigma, 11)
        q = mixture(40, d, nc, sigma, 12)
        idx = ref.ivfpq()
        idx.train(x[:nt], nlist, m, 8, use_opq=opq, brute_assign=True, opq_sample_n=1200)
        # An empty index (trained model only) for add parity.
        out_model = os.path.join(HERE, f"ivfpq_{name}_model")
        shutil.rmtree(out_model, ignore_errors=True)
        idx.save(out_model)
        idx.add(np.arange(nb, dtype=np.uint64) * 3 + 7, x)
        out = os.path.join(HERE, f"ivfpq_{name}")
        shutil.rmtree(out, ignore_errors=True)
        idx.save(out)
        res = {}
        for k, npb in SEARCHES:
            ids, dist, cnt = idx.search(q, k, npb)
            res[f"ids_{k}_{npb}"] = ids
            res[f"d_{k}_{npb}"] = dist
            res[f"n_{k}_{npb}"] = cnt
        np.savez_compressed(os.path.join(HERE, f"ivfpq_{name}.npz"), base=x, queries=q, n_train=nt, **res)
        print("wrote", name)


# (k, nprobe, cand_k, rerank_k) searches with the exact rerank on
RERANK_SEARCHES = [(10, 8, 0, 0), (5, 16, 0, 20), (10, 4, 50, 30), (3, 64, 0, 2), (20, 8, 100, 0)]


def make_rerank(ref: Reference):
    """The reference's exact rerank (IvfPqSearchParams::use_exact_rerank) on the saved
    golden indexes: ivfpq_<case>_rerank.npz."""
    for (name, *_rest) in CASES:
        data = np.load(os.path.join(HERE, f"ivfpq_{name}.npz"))
        idx = ref.ivfpq()
        idx.load(os.path.join(HERE, f"ivfpq_{name}"))
        res = {}
        for k, npb, ck, rk in RERANK_SEARCHES:
            ids, dist, cnt = idx.search(data["queries"], k, npb, cand_k=ck, rerank=True, rerank_k=rk)
            tag = f"{k}_{npb}_{ck}_{rk}"
            res[f"ids_{tag}"], res[f"d_{tag}"], res[f"n_{tag}"] = ids, dist, cnt
        np.savez_compressed(os.path.join(HERE, f"ivfpq_{name}_rerank.npz"), **res)
        print("wrote", name, "rerank")


def make_api(ref: Reference):
    """The rest of IvfPqIndex's API on the saved golden indexes (ivfpq_<case>_api.npz):
    reconstruct / get_cluster_assignment of some ids (including a missing one),
    reconstruct_cluster of a few clusters, the debug rank explanations (which need
    VESPER_IVFPQ_DEBUG=1), then update_cluster_centroid + reassign_vector, saved again
    (ivfpq_<case>_api/ivfpq.bin)."""
    os.environ["VESPER_IVFPQ_DEBUG"] = "1"
    for (name, d, nlist, *_rest) in CASES:
        data = np.load(os.path.join(HERE, f"ivfpq_{name}.npz"))
        idx = ref.ivfpq()
        idx.load(os.path.join(HERE, f"ivfpq_{name}"))
        nb = data["base"].shape[0]
        ids = (np.array([0, 1, 5, nb // 2, nb - 1], dtype=np.uint64) * 3 + 7).tolist() + [2]  # 2: not an id
        res = {"ids": np.array(ids, np.uint64)}
        rec, rc_rec, asg, rc_asg = [], [], [], []
        for vid in ids:
            rc, v = idx.reconstruct(vid, d)
            rec.append(v); rc_rec.append(rc)
            rc, a = idx.get_cluster_assignment(vid)
            asg.append(a); rc_asg.append(rc)
        res.update(reconstruct=np.array(rec), reconstruct_rc=np.array(rc_rec), assign=np.array(asg, np.uint32),
                   assign_rc=np.array(rc_asg))
        for c in (0, nlist // 2, nlist - 1):
            rc, cids, vec = idx.reconstruct_cluster(c, d)
            res[f"cluster_{c}_ids"], res[f"cluster_{c}_vec"], res[f"cluster_{c}_rc"] = cids, vec, rc
        rc, _, _ = idx.reconstruct_cluster(nlist, d)
        res["cluster_bad_rc"] = rc
        q = data["queries"][:4]
        cr, ar = [], []
        for i, vid in enumerate(ids[:4]):
            rc, rank, cl = idx.debug_centroid_rank(q[i], vid)
            cr.append((rc, rank, cl))
            rc, rank, dist = idx.debug_adc_rank(q[i], vid)
            ar.append((rc, rank, dist))
        res["centroid_rank"] = np.array(cr, np.float64)
        res["adc_rank"] = np.array(ar, np.float64)
        # mutations: a centroid moved, then three vectors reassigned
        g = np.random.default_rng(5)
        newc = g.standard_normal(d).astype(np.float32)
        res["update_cluster"], res["update_centroid"] = np.uint32(1), newc
        res["update_rc"] = idx.update_cluster_centroid(1, newc)
        moves = [(ids[0], nlist - 1), (ids[2], 0), (ids[3], 1)]
        res["moves"] = np.array(moves, np.uint64)
        res["move_rc"] = np.array([idx.reassign_vector(v, c) for v, c in moves])
        out = os.path.join(HERE, f"ivfpq_{name}_api")
        shutil.rmtree(out, ignore_errors=True)
        idx.save(out)
        np.savez_compressed(os.path.join(HERE, f"ivfpq_{name}_api.npz"), **res)
        print("wrote", name, "api")


V11_CASES = [("plain_d32_m8", '{"name": "golden", "tags": ["a", "b"], "n": 2000, "nested": {"x": [1.5e3, null, true]}}'),
             ("opq_d32_m4", "")]
BAD_METADATA = ['{"a": 1', '{"a": 1} x', '[' * 65 + ']' * 65, '{"a": "\\q"}']


def make_v11(ref: Reference):
    """The golden indexes re-saved by the reference with VESPER_IVFPQ_SAVE_V11=1."""
    os.environ["VESPER_IVFPQ_SAVE_V11"] = "1"
    rec = {"metadata": {}, "bad_metadata": []}
    try:
        for name, meta in V11_CASES:
            idx = ref.ivfpq()
            idx.load(os.path.join(HERE, f"ivfpq_{name}"))
            if meta:
                idx.set_metadata_json(meta)
            out = os.path.join(HERE, f"ivfpq_{name}_v11")
            shutil.rmtree(out, ignore_errors=True)
            idx.save(out)
            back = ref.ivfpq()
            back.load(out)
            assert back.get_metadata_json() == meta
            rec["metadata"][name] = meta
            print("wrote", name, "v11")
        with __import__("tempfile").TemporaryDirectory() as td:
            for bad in BAD_METADATA:
                idx = ref.ivfpq()
                idx.load(os.path.join(HERE, f"ivfpq_{V11_CASES[0][0]}"))
                idx.set_metadata_json(bad)
                try:
                    idx.save(td)
                    msg = ""
                except IOError as e:
                    msg = str(e)
                rec["bad_metadata"].append([bad, msg])
    finally:
        os.environ.pop("VESPER_IVFPQ_SAVE_V11", None)
    with open(os.path.join(HERE, "ivfpq_v11.json"), "w") as f:
        json.dump(rec, f, indent=1)


def make_kmeans(ref: Reference):
    x = mixture(3000, 16, 60, 0.05, 21)
    kpp = ref.kmeanspp_init(x, 48, 42)
    c_e, a_e, it_e, in_e = ref.kmeans_elkan(x, 48, 25, 1e-4, 42)
    c_l, a_l, it_l, in_l = ref.kmeans_lloyd(x, 48, 20, 0.0, 42)
    asg, inert = ref.kmeans_assign(x, kpp)
    upd = ref.kmeans_update(x, asg, kpp)
    pq = ref.pq(4, 8)
    pq.train(x)
    np.savez_compressed(os.path.join(HERE, "kmeans_small.npz"), x=x, kpp=kpp, elkan_c=c_e, elkan_a=a_e,
                        elkan_it=it_e, elkan_inertia=in_e, lloyd_c=c_l, lloyd_a=a_l, lloyd_it=it_l,
                        lloyd_inertia=in_l, assign=asg, assign_inertia=inert, update=upd,
                        pq_cb=pq.codebooks())
    print("wrote kmeans_small")


if __name__ == "__main__":
    args = [a for a in sys.argv[1:] if not a.startswith("--")]
    ref_root = args[0] if args else os.environ.get("VESPER_REFERENCE_DIR")
    if not ref_root:
        sys.exit("usage: make_golden.py <reference source root> (or set VESPER_REFERENCE_DIR)")
    convert_fixtures(ref_root)
    ref = Reference()
    only = [a for a in sys.argv if a.endswith("-only")]
    if not only:
        make_ivfpq(ref)
        make_kmeans(ref)
    if not only or "--rerank-only" in only:
        make_rerank(ref)
    if not only or "--api-only" in only:
        make_api(ref)
    if not only or "--v11-only" in only:
        make_v11(ref)
