"""The CPU sum-tree baseline against vectors produced by the reference itself.

tests/golden/sumtree_small.npz was made by tests/golden/make_golden.py, which
runs triton-per's own CpuSumTreePER (src/triton_per/baselines/cpu_sumtree.py)
on the seeded inputs of cases.case_sumtree(): a store of 1000 slots (not a
power of two) filled past one lap, updates with duplicate indices, samples of
512 draws. The C restatement (oracle/per_sumtree.c) and the plain-Python one
(oracle/sumtree.PySumTree) must reproduce the float64 tree bit for bit, the
sampled indices and rows exactly, and the float32 weights to one ulp (numpy's
vectorised pow against glibc's pow).
"""

import os

import numpy as np
import pytest

import cases
from oracle import sumtree

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "sumtree_small.npz")


def ulps(a, b):
    a = np.asarray(a, np.float32).view(np.int32).astype(np.int64)
    b = np.asarray(b, np.float32).view(np.int32).astype(np.int64)
    return np.abs(a - b)


@pytest.fixture(scope="module")
def golden():
    g = np.load(GOLDEN)
    c = cases.case_sumtree()
    assert str(g["inputs_digest"]) == cases.sumtree_inputs_digest(c), "case inputs drifted"
    return c, g


def test_c_sumtree_matches_reference(golden):
    c, g = golden
    st = sumtree.SumTreeStore(c["capacity"], 3)
    for k in range(2):
        st.add(c["adds"][k])
        np.testing.assert_array_equal(st.tree, g[f"s{k}_tree_after_add"])
        st.update_priorities(c["upd_idx"][k], c["upd_td"][k])
        np.testing.assert_array_equal(st.tree, g[f"s{k}_tree"])
        assert st.max_priority == float(g[f"s{k}_max_priority"])
        assert [st.cursor, st.size] == g[f"s{k}_cursor_size"].tolist()
        idx, w = st.sample_from_uniforms(c["rand"][k], c["beta"])
        np.testing.assert_array_equal(idx, g[f"s{k}_idx"])
        assert ulps(w, g[f"s{k}_w"]).max() <= 1
        np.testing.assert_array_equal(st.gather(idx), g[f"s{k}_rows"])


def test_python_sumtree_matches_reference(golden):
    c, g = golden
    st = sumtree.PySumTree(c["capacity"], 3)
    cursor = 0
    for k in range(2):
        rows = c["adds"][k]
        for j in range(rows.shape[0]):  # cpu_sumtree.py:64-73
            i = (cursor + j) % c["capacity"]
            st.update(i, st.max_priority)
            st.storage[i] = rows[j]
        cursor = (cursor + rows.shape[0]) % c["capacity"]
        st.size = min(st.size + rows.shape[0], c["capacity"])
        np.testing.assert_array_equal(st.tree, g[f"s{k}_tree_after_add"])
        st.update_priorities(c["upd_idx"][k], c["upd_td"][k])
        np.testing.assert_array_equal(st.tree, g[f"s{k}_tree"])
        idx, w, out = st.sample_from_uniforms(c["rand"][k], c["beta"])
        np.testing.assert_array_equal(idx, g[f"s{k}_idx"])
        assert ulps(w, g[f"s{k}_w"]).max() <= 1
        np.testing.assert_array_equal(out, g[f"s{k}_rows"])


def test_build_from_leaves_gives_the_same_sums():
    """The bench's set-up shortcut: leaves written at once equal, sum for sum,
    a tree whose leaves were set one update() at a time (exact for leaves that
    are sums of few binary digits; here small dyadic values)."""
    rng = np.random.default_rng(0)
    cap = 777
    leaves = rng.integers(1, 64, cap).astype(np.float64) / 8.0
    a = sumtree.SumTreeStore(cap, 1)
    a.build_from_leaves(leaves)
    b = sumtree.PySumTree(cap, 1)
    for i, v in enumerate(leaves):
        b.update(i, float(v))
    np.testing.assert_array_equal(a.tree[1:], b.tree[1:])
    u = rng.random(1000) * a.total()
    found = [sumtree.lib().sumtree_find(a.tree, cap, float(x)) for x in u]
    assert found == [b.find(float(x)) for x in u]
