"""The rest of IvfPqIndex's API on the GPU index against the reference's own results.

reconstruct / get_cluster_assignment / reconstruct_cluster / debug_explain_* on the
golden indexes, then update_cluster_centroid + reassign_vector: the lists they leave must
equal those the reference saved after the same calls (tests/golden/ivfpq_<case>_api),
and searches on the changed index must match the oracle.  compact_inverted_list is
checked against its definition (entries whose 32-bit id is in the set leave the list).
"""
import os

import numpy as np
import pytest

from conftest import CASES, GOLDEN, SEARCHES, assert_topk_equivalent, golden_case

pytestmark = pytest.mark.gpu


def _index():
    from vesper_db_b200 import IvfPqIndex
    return IvfPqIndex()


@pytest.mark.parametrize("name", CASES)
def test_index_api_matches_reference(name, oracle, monkeypatch):
    from oracle_lib import read_ivfpq_v10

    from vesper_db_b200 import SEARCH_EXACT, VesperError
    monkeypatch.setenv("VESPER_IVFPQ_DEBUG", "1")
    f, _, data = golden_case(name)
    g = np.load(os.path.join(GOLDEN, f"ivfpq_{name}_api.npz"))
    idx = _index()
    idx.load(os.path.join(GOLDEN, f"ivfpq_{name}"))
    nlist = f["centroids"].shape[0]
    for i, vid in enumerate(g["ids"]):
        if g["reconstruct_rc"][i] == 6001:
            with pytest.raises(VesperError, match="not found"):
                idx.reconstruct(int(vid))
            with pytest.raises(VesperError, match="not found"):
                idx.get_cluster_assignment(int(vid))
            continue
        assert np.array_equal(idx.reconstruct(int(vid)), g["reconstruct"][i])
        assert idx.get_cluster_assignment(int(vid)) == g["assign"][i]
    for c in (0, nlist // 2, nlist - 1):
        ids, vec = idx.reconstruct_cluster(c)
        assert np.array_equal(ids, g[f"cluster_{c}_ids"])
        assert np.array_equal(vec.reshape(-1), g[f"cluster_{c}_vec"].reshape(-1))
    with pytest.raises(VesperError, match="Invalid cluster ID"):
        idx.reconstruct_cluster(nlist)
    q = data["queries"][:4]
    for i in range(4):
        vid = int(g["ids"][i])
        assert idx.debug_explain_centroid_rank(q[i], vid) == (int(g["centroid_rank"][i][1]),
                                                             int(g["centroid_rank"][i][2]))
        rank, dist = idx.debug_explain_adc_rank(q[i], vid)
        assert rank == int(g["adc_rank"][i][1]) and np.float32(dist) == np.float32(g["adc_rank"][i][2])
    # the reference's mutations, then the lists it saved
    idx.update_cluster_centroid(int(g["update_cluster"]), g["update_centroid"])
    assert np.array_equal(idx.get_cluster_centroid(int(g["update_cluster"])), g["update_centroid"])
    for vid, c in g["moves"]:
        idx.reassign_vector(int(vid), int(c))
    f2 = read_ivfpq_v10(os.path.join(GOLDEN, f"ivfpq_{name}_api", "ivfpq.bin"))
    offs, ids, codes = idx.lists()
    assert np.array_equal(offs, f2["list_offsets"])
    assert np.array_equal(ids, f2["ids"]) and np.array_equal(codes, f2["codes"])
    # searches on the changed index: EXACT bit-exact, FAST within tolerance
    for k, npb in SEARCHES[:3]:
        rids, rd, rcnt = oracle.ivfpq_search(data["queries"], f2["centroids"], f2["rotation"], f2["codebooks"],
                                             f2["m"], f2["list_offsets"], f2["ids"], f2["codes"], k, npb)
        gi, gd, gn = idx.search_batch(data["queries"], k, npb, mode=SEARCH_EXACT)
        assert_topk_equivalent(gi, gd, gn, rids, rd, rcnt, 0.0)
        gi, gd, gn = idx.search_batch(data["queries"], k, npb)
        assert_topk_equivalent(gi, gd, gn, rids, rd, rcnt, 1e-4)


def test_debug_explain_requires_the_debug_switch(monkeypatch):
    from vesper_db_b200 import VesperError
    monkeypatch.delenv("VESPER_IVFPQ_DEBUG", raising=False)
    f, _, data = golden_case(CASES[0])
    idx = _index()
    idx.load(os.path.join(GOLDEN, f"ivfpq_{CASES[0]}"))
    with pytest.raises(VesperError, match="VESPER_IVFPQ_DEBUG"):
        idx.debug_explain_adc_rank(data["queries"][0], 7)


def test_compact_inverted_list(oracle):
    from vesper_db_b200 import SEARCH_EXACT, VesperError
    f, _, data = golden_case(CASES[1])
    idx = _index()
    idx.load(os.path.join(GOLDEN, f"ivfpq_{CASES[1]}"))
    offs, ids, codes = idx.lists()
    c = int(np.argmax(np.diff(offs.astype(np.int64))))
    members = ids[offs[c]:offs[c + 1]]
    gone = np.concatenate([members[::3], np.array([1, 2, 3], np.uint64)])  # plus ids not in the list
    removed = idx.compact_inverted_list(c, gone.astype(np.uint32))
    keep = np.ones(ids.shape[0], bool)
    keep[offs[c]:offs[c + 1]] = ~np.isin(members, members[::3])
    assert removed == int((~keep).sum())
    offs2, ids2, codes2 = idx.lists()
    assert np.array_equal(ids2, ids[keep]) and np.array_equal(codes2, codes[keep])
    exp_offs = offs.copy()
    exp_offs[c + 1:] -= removed
    assert np.array_equal(offs2, exp_offs)
    assert idx.get_stats()["n_vectors"] == ids2.shape[0]
    rids, rd, rcnt = oracle.ivfpq_search(data["queries"], f["centroids"], f["rotation"], f["codebooks"], f["m"],
                                         offs2, ids2, codes2, 10, 8)
    gi, gd, gn = idx.search_batch(data["queries"], 10, 8, mode=SEARCH_EXACT)
    assert_topk_equivalent(gi, gd, gn, rids, rd, rcnt, 0.0)
    with pytest.raises(VesperError, match="out of range"):
        idx.compact_inverted_list(f["centroids"].shape[0], [1])
