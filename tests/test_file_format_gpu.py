"""The index file formats (IvfPqIndex::save / load, src/index/ivf_pq.cpp:4241-4966).

v1.0 is the monolithic layout; v1.1 (written with VESPER_IVFPQ_SAVE_V11=1) stores the
centroids, codebooks, OPQ rotation, JSON metadata and inverted lists as checksummed
sections.  The loader reads both; the writer must reproduce the reference's bytes
exactly, except the build timestamp (header bytes 48..56) and so the file checksum.
"""
import json
import os
import struct
import tempfile

import numpy as np
import pytest

from conftest import GOLDEN, assert_topk_equivalent, golden_case

pytestmark = pytest.mark.gpu

V11 = json.load(open(os.path.join(GOLDEN, "ivfpq_v11.json")))
TS = slice(48, 56)


def _index():
    from vesper_db_b200 import IvfPqIndex
    return IvfPqIndex()


def _fnv(b: bytes) -> int:
    h = 1469598103934665603
    for x in b:
        h = ((h ^ x) * 1099511628211) & 0xFFFFFFFFFFFFFFFF
    return h


def _write(path, body: bytes):
    os.makedirs(path, exist_ok=True)
    with open(os.path.join(path, "ivfpq.bin"), "wb") as f:
        f.write(body + b"CHKS" + struct.pack("<Q", _fnv(body)))


def _same_but_timestamp(a: bytes, b: bytes):
    assert len(a) == len(b)
    assert a[:TS.start] == b[:TS.start]
    assert a[TS.stop:-8] == b[TS.stop:-8]


@pytest.mark.parametrize("name", ["plain_d32_m8", "opq_d32_m4"])
def test_load_v11_matches_v10(name):
    f, _, data = golden_case(name)
    a, b = _index(), _index()
    a.load(os.path.join(GOLDEN, f"ivfpq_{name}"))
    b.load(os.path.join(GOLDEN, f"ivfpq_{name}_v11"))
    assert b.get_metadata_json() == V11["metadata"][name]
    for x, y in zip(a.lists(), b.lists()):
        assert np.array_equal(x, y)
    from vesper_db_b200 import SEARCH_EXACT
    for k, npb in [(10, 4), (100, 8)]:
        ra = a.search_batch(data["queries"], k, npb, mode=SEARCH_EXACT)
        rb = b.search_batch(data["queries"], k, npb, mode=SEARCH_EXACT)
        for x, y in zip(ra, rb):
            assert np.array_equal(x, y)
        assert_topk_equivalent(*rb, data[f"ids_{k}_{npb}"], data[f"d_{k}_{npb}"], data[f"n_{k}_{npb}"], 0.0)


@pytest.mark.parametrize("name", ["plain_d32_m8", "opq_d32_m4"])
def test_save_v11_reproduces_reference_bytes(name):
    idx = _index()
    idx.load(os.path.join(GOLDEN, f"ivfpq_{name}"))
    if V11["metadata"][name]:
        idx.set_metadata_json(V11["metadata"][name])
    ref_bytes = open(os.path.join(GOLDEN, f"ivfpq_{name}_v11", "ivfpq.bin"), "rb").read()
    with tempfile.TemporaryDirectory() as td:
        os.environ["VESPER_IVFPQ_SAVE_V11"] = "1"
        try:
            idx.save(td)
        finally:
            os.environ.pop("VESPER_IVFPQ_SAVE_V11", None)
        got = open(os.path.join(td, "ivfpq.bin"), "rb").read()
        _same_but_timestamp(got, ref_bytes)
        again = _index()
        again.load(td)
        assert again.get_metadata_json() == V11["metadata"][name]


@pytest.mark.parametrize("name", ["plain_d32_m8", "opq_d32_m4"])
def test_save_v10_reproduces_reference_bytes(name):
    idx = _index()
    idx.load(os.path.join(GOLDEN, f"ivfpq_{name}"))
    idx.set_metadata_json('{"ignored": "by v1.0"}')
    ref_bytes = open(os.path.join(GOLDEN, f"ivfpq_{name}", "ivfpq.bin"), "rb").read()
    with tempfile.TemporaryDirectory() as td:
        idx.save(td)
        _same_but_timestamp(open(os.path.join(td, "ivfpq.bin"), "rb").read(), ref_bytes)


def test_invalid_metadata_refused_as_the_reference_does():
    from vesper_db_b200 import VesperError
    idx = _index()
    idx.load(os.path.join(GOLDEN, "ivfpq_plain_d32_m8"))
    with tempfile.TemporaryDirectory() as td:
        os.environ["VESPER_IVFPQ_SAVE_V11"] = "1"
        try:
            for bad, msg in V11["bad_metadata"]:
                idx.set_metadata_json(bad)
                with pytest.raises(VesperError) as e:
                    idx.save(td)
                assert msg in str(e.value)
        finally:
            os.environ.pop("VESPER_IVFPQ_SAVE_V11", None)


def test_v11_corruption_and_unknown_sections():
    """A flipped payload byte fails the file checksum; a flipped byte with the file
    checksum recomputed fails the section checksum; an unknown section type is
    skipped; an empty section header is skipped; a truncated inverted section and a
    compressed section are refused."""
    from vesper_db_b200 import VesperError
    src = open(os.path.join(GOLDEN, "ivfpq_plain_d32_m8_v11", "ivfpq.bin"), "rb").read()
    body = src[:-12]
    hdr = 60 + 0  # fixed header with meta_len = 0
    f, _, data = golden_case("plain_d32_m8")
    with tempfile.TemporaryDirectory() as td:
        bad = bytearray(src)
        bad[hdr + 28 + 5] ^= 1          # inside the centroid payload
        os.makedirs(td, exist_ok=True)
        open(os.path.join(td, "ivfpq.bin"), "wb").write(bytes(bad))
        with pytest.raises(VesperError, match="Checksum mismatch"):
            _index().load(td)
        _write(td, bytes(bad[:-12]))
        with pytest.raises(VesperError, match="Section checksum mismatch"):
            _index().load(td)
        # an unknown section (type 77) and an empty section after the header
        extra = struct.pack("<IQQQ", 77, 5, 5, _fnv(b"hello")) + b"hello" + struct.pack("<IQQQ", 2, 0, 0, 0)
        _write(td, body[:hdr] + extra + body[hdr:])
        idx = _index()
        idx.load(td)
        from vesper_db_b200 import SEARCH_EXACT
        res = idx.search_batch(data["queries"], 10, 4, mode=SEARCH_EXACT)
        assert_topk_equivalent(*res, data["ids_10_4"], data["d_10_4"], data["n_10_4"], 0.0)
        # the inverted section is last: drop its final byte and fix its header
        inv_start = body.rfind(struct.pack("<I", 3), 0)
        while True:
            unc = struct.unpack_from("<Q", body, inv_start + 4)[0]
            if inv_start + 28 + unc == len(body):
                break
            inv_start = body.rfind(struct.pack("<I", 3), 0, inv_start)
        payload = body[inv_start + 28:-1]
        trunc = body[:inv_start] + struct.pack("<IQQQ", 3, len(payload), len(payload), _fnv(payload)) + payload
        _write(td, trunc)
        with pytest.raises(VesperError, match="Entry truncated|Inverted section extra bytes"):
            _index().load(td)
        comp = body[:hdr] + struct.pack("<IQQQ", 9, 100, 5, 0) + b"xxxxx" + body[hdr:]
        _write(td, comp)
        with pytest.raises(VesperError, match="Decompression failed"):
            _index().load(td)


def test_reference_loads_our_v11_file(reference):
    f, _, data = golden_case("opq_d32_m4")
    idx = _index()
    idx.load(os.path.join(GOLDEN, "ivfpq_opq_d32_m4"))
    idx.set_metadata_json('{"from": "gpu"}')
    with tempfile.TemporaryDirectory() as td:
        os.environ["VESPER_IVFPQ_SAVE_V11"] = "1"
        try:
            idx.save(td)
        finally:
            os.environ.pop("VESPER_IVFPQ_SAVE_V11", None)
        r = reference.ivfpq()
        r.load(td)
        assert r.get_metadata_json() == '{"from": "gpu"}'
