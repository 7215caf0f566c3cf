import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden")
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "oracle"))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); run with -m gpu")


CASES = ["plain_d32_m8", "plain_d64_m8", "opq_d32_m4", "odd_d20_m5", "plain_d64_n128"]
SEARCHES = [(10, 4), (10, 16), (100, 8), (5, 1), (3, 64)]


@pytest.fixture(scope="session")
def oracle():
    from oracle_lib import Oracle
    return Oracle()


@pytest.fixture(scope="session")
def reference():
    from oracle_lib import REF_NC_SO, Reference
    if not os.path.exists(REF_NC_SO):
        pytest.skip("oracle/_ref not built here (the reference sources are not mounted)")
    return Reference()


def golden_case(name):
    from oracle_lib import read_ivfpq_v10
    f = read_ivfpq_v10(os.path.join(GOLDEN, f"ivfpq_{name}", "ivfpq.bin"))
    model = read_ivfpq_v10(os.path.join(GOLDEN, f"ivfpq_{name}_model", "ivfpq.bin"))
    data = dict(np.load(os.path.join(GOLDEN, f"ivfpq_{name}.npz")))
    return f, model, data


def assert_topk_equivalent(ids, d, cnt, ref_ids, ref_d, ref_cnt, rtol):
    """Distances within rtol (relative, floor 1) position by position; the id sets equal
    except for ties at the k-th distance: an id that only one side returns must lie, on
    that side, within rtol of the reference's k-th distance."""
    ids, d, ref_ids, ref_d = map(np.asarray, (ids, d, ref_ids, ref_d))
    assert np.array_equal(np.asarray(cnt), np.asarray(ref_cnt)), "result counts differ"
    for q in range(ids.shape[0]):
        n = int(ref_cnt[q])
        if n == 0:
            continue
        a, b = d[q, :n].astype(np.float64), ref_d[q, :n].astype(np.float64)
        tol = rtol * np.maximum(1.0, np.abs(b))
        assert np.all(np.abs(a - b) <= tol), \
            f"query {q}: distances differ beyond {rtol}: max {np.abs(a - b).max()} at {int(np.argmax(np.abs(a - b)))}"
        kth = b[n - 1]
        band = rtol * max(1.0, abs(kth))
        ia, ib = [int(i) for i in ids[q, :n]], [int(i) for i in ref_ids[q, :n]]
        sa, sb = set(ia), set(ib)
        off = [(i, float(x), "ours") for i, x in zip(ia, a) if i not in sb and abs(x - kth) > band]
        off += [(i, float(x), "reference") for i, x in zip(ib, b) if i not in sa and abs(x - kth) > band]
        assert not off, f"query {q}: ids returned by one side only, away from the k-th distance {kth}: {off}"
