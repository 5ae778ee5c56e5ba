"""The oracle against vectors produced by the reference itself (CPU only).

tests/golden/*.npz were made by tests/golden/make_golden.py, which runs
triton-per's own torch backend (src/triton_per/buffer.py) on the seeded inputs
of tests/golden/cases.py. Indices must be bit-exact; float32 values that come
from pow may differ by one ulp between glibc and torch's vectorised pow.
"""

import os

import numpy as np
import pytest

import cases
from oracle import oracle

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def load(name):
    return np.load(os.path.join(GOLDEN, name + ".npz"))


def ulps(a, b):
    a = np.asarray(a, np.float32).view(np.int32).astype(np.int64)
    b = np.asarray(b, np.float32).view(np.int32).astype(np.int64)
    return np.abs(a - b)


@pytest.mark.parametrize("name", sorted(cases.SAMPLE_CASES))
def test_oracle_sample_matches_reference(name):
    c = cases.SAMPLE_CASES[name]()
    g = load("sample_" + name)
    assert str(g["inputs_digest"]) == cases.sample_inputs_digest(c), "case inputs drifted"
    leaves = np.zeros(-(-c["capacity"] // 1024) * 1024, np.float32)
    leaves[: c["leaves"].size] = c["leaves"]
    idx, w, csum = oracle.sample(leaves, c["capacity"], c["size"], c["rand"], c["beta"])
    assert csum[-1] == g["total"]
    np.testing.assert_array_equal(idx, g["idx"])
    assert ulps(w, g["w"]).max() <= 2
    np.testing.assert_allclose(w, g["w"], rtol=1e-6, atol=0)
    rows = np.concatenate([c["rows"][k] for k in c["fields"]], axis=1)
    assert cases.digest(rows[idx]) == str(g["out_digest"])


def test_oracle_config1_update_then_sample():
    c = cases.case_config1()
    g = load("sample_config1")
    st = oracle.OracleStore(c["capacity"], c["fields"])
    st.add(c["rows"])
    st.set_priorities(np.pad(c["leaves"], (0, st.capacity_padded - c["capacity"])))
    idx, w, _ = st.sample_from_uniforms(c["rand"], c["beta"])
    np.testing.assert_array_equal(idx, g["idx"])
    upd = cases.dup_indices(c["dup_rng"], idx, c["dup_frac"])
    np.testing.assert_array_equal(upd, g["upd_idx"])
    assert 0 < (upd.size - np.unique(upd).size) <= 40  # ~10% duplicates
    st.update_priorities(upd, c["td"])
    assert ulps(st.priorities[g["upd_uniq"]], g["upd_leaves"]).max() <= 1
    np.testing.assert_allclose(st.block_sums, g["upd_block_sums"], rtol=1e-6)
    assert ulps(st.max_priority, g["upd_max_priority"]).max() <= 1
    idx2, w2, _ = st.sample_from_uniforms(c["rand2"], c["beta"])
    np.testing.assert_array_equal(idx2, g["idx2"])
    np.testing.assert_allclose(w2, g["w2"], rtol=1e-6)


@pytest.mark.parametrize("name,fn", [("update_dups", cases.case_update_dups),
                                     ("update_storm", cases.case_update_storm)])
def test_oracle_update_matches_reference(name, fn):
    c = fn()
    g = load(name)
    assert str(g["inputs_digest"]) == cases.digest(c["leaves"], c["idx"], c["td"])
    nb = -(-c["capacity"] // 1024)
    leaves = np.zeros(nb * 1024, np.float32)
    leaves[: c["capacity"]] = c["leaves"]
    bs = oracle.block_sums(leaves)
    mp = np.float32(1.0)
    st = oracle.OracleStore(c["capacity"], {"x": 1}, alpha=c["alpha"], eps=c["eps"])
    st.set_priorities(leaves)
    st.update_priorities(c["idx"], c["td"])
    assert ulps(st.priorities, g["leaves"]).max() <= 1
    np.testing.assert_allclose(st.block_sums, g["block_sums"], rtol=1e-6)
    assert ulps(st.max_priority, g["max_priority"]).max() <= 1
    del bs, mp


def test_oracle_add_wraparound_matches_reference():
    c = cases.case_add_wrap()
    g = load("add_wrap")
    st = oracle.OracleStore(c["capacity"], c["fields"])
    steps = [("add", c["adds"][0]), ("upd", None), ("add", c["adds"][1]), ("add", c["adds"][2])]
    for k, (kind, rows) in enumerate(steps):
        if kind == "add":
            st.add({"x": rows})
        else:
            st.update_priorities(c["upd_idx"], c["upd_td"])
        np.testing.assert_array_equal(st.storage, g[f"s{k}_storage"])
        assert ulps(st.priorities, g[f"s{k}_leaves"]).max() <= 1
        np.testing.assert_allclose(st.block_sums, g[f"s{k}_block_sums"], rtol=1e-6)
        np.testing.assert_array_equal([st.cursor, st.size], g[f"s{k}_cursor_size"])
        assert ulps(st.max_priority, g[f"s{k}_max_priority"]).max() <= 1


def test_ties_case_really_has_ties():
    """The tie case must exercise u == prefix: right=True picks the next slot."""
    c = cases.case_ties()
    csum = oracle.cumsum(c["leaves"])
    u = (c["rand"] * csum[-1]).astype(np.float32)
    hits = np.isin(u, csum).sum()
    assert hits > 1000


def test_classifier_excuses_only_boundary_ties():
    c = cases.case_ties()
    cap = c["capacity"]
    leaves = np.zeros(3072, np.float32)
    leaves[:cap] = c["leaves"]
    idx, _, csum = oracle.sample(leaves, cap, cap, c["rand"], 0.5)
    csum = csum[:cap]
    u = (c["rand"] * csum[-1]).astype(np.float32)
    # a searcher that breaks ties the other way (first prefix >= u)
    left = np.minimum(np.searchsorted(csum, u, side="left"), cap - 1)
    eq, exc, bad = oracle.classify_indices(left, idx, c["rand"], csum, cap)
    assert exc > 1000 and bad.size == 0 and eq + exc == idx.size
    # an off-by-one everywhere is NOT excused
    wrong = np.minimum(idx + 1, cap - 1)
    _, _, bad2 = oracle.classify_indices(wrong, idx, c["rand"], csum, cap)
    assert bad2.size > 1000


def test_philox_known_answers():
    """The oracle's Philox4x32-10 against the published known-answer vectors
    of the generator's authors (Random123 kat_vectors: zero, all-ones and pi
    digits counter/key)."""
    from oracle import oracle

    kat = [
        ((0, 0, 0, 0), (0, 0), (0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8)),
        ((0xFFFFFFFF,) * 4, (0xFFFFFFFF, 0xFFFFFFFF), (0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD)),
        ((0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344), (0xA4093822, 0x299F31D0),
         (0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1)),
    ]
    for ctr, key, want in kat:
        got = oracle.philox4x32_10(np.array([ctr], np.uint64), key)[0]
        assert tuple(int(x) for x in got) == want
    u = oracle.philox_uniforms(12345, 2**32 - 3, 10)  # counter crosses the 32-bit boundary
    assert u.dtype == np.float32 and ((u >= 0) & (u < 1)).all()
