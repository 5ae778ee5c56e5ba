"""The update paths against the oracle (B200).

Batches of up to 2048 indices go through the partitioned update (CTAs owning
disjoint top-level nodes, each applying its entries in rounds of 32 with warp
elections); larger batches take the grid path. Every path must give the
oracle's leaves (last occurrence wins, within 1e-6) and exact tree sums, on
trees of 2, 3 and 4 levels. The sharded entry point with a device count
applies only the counted prefix of its indices."""

import ctypes

import numpy as np
import pytest
import torch

import cases
from helpers import SUM_RTOL, check_tree, make_buffer
from oracle import oracle
from per_b200 import _lib

pytestmark = pytest.mark.gpu


def _dup_batch(rng, cap, n):
    half = rng.integers(0, cap, (n + 1) // 2)
    idx = np.concatenate([half, half[rng.integers(0, half.size, n - half.size)]])
    rng.shuffle(idx)
    td = (rng.standard_normal(n) * 3).astype(np.float32)
    return idx.astype(np.int64), td


@pytest.mark.parametrize("cap,n", [(1_000_000, 1), (1_000_000, 32), (1_000_000, 256),
                                   (1_000_000, 512), (100_000, 300), (20_000, 500),
                                   (20_000, 2048), (5_000_000, 400), (5_000_000, 2049),
                                   (1_000_000, 300), (1_000_000, 513), (1_000_000, 2048), (1_000_000, 1024),
                                   (1_000_000, 2500), (1_000_000, 4096), (1_000_000, 5000),
                                   (5_000_000, 700), (5_000_000, 3000)])
def test_update_matches_oracle(cap, n):
    rng = np.random.default_rng(cap // 1000 + n)
    leaves = cases.leaves_abs_normal(rng, cap)
    buf = make_buffer(cap, {"x": 1}, None, leaves)
    st = oracle.OracleStore(cap, {"x": 1})
    lv = np.zeros(st.capacity_padded, np.float32)
    lv[:cap] = leaves
    st.set_priorities(lv)
    for _ in range(2):  # twice: the second call finds the first one's tree
        idx, td = _dup_batch(rng, cap, n)
        buf.update_priorities(torch.from_numpy(idx).cuda(), torch.from_numpy(td).cuda())
        st.update_priorities(idx, td)
    np.testing.assert_allclose(buf.priorities.cpu().numpy()[:cap], st.priorities[:cap],
                               rtol=1e-6, atol=0)
    check_tree(buf)
    assert buf._max_priority.item() == pytest.approx(float(st.max_priority), rel=1e-6)
    s = buf.status()
    assert s["errors"] == 0 and s["timeouts"] == 0


@pytest.mark.parametrize("n,count", [(400, 150), (512, 512), (256, 0), (600, 250),
                                     (2048, 2048), (2048, 0), (2048, 1999), (4096, 1500)])
def test_shard_update_reads_only_the_counted_prefix(n, count):
    rng = np.random.default_rng(n + count)
    cap, base = 200_000, 400_000
    leaves = cases.leaves_abs_normal(rng, cap)
    buf = make_buffer(cap, {"x": 1}, None, leaves)
    gidx, td = _dup_batch(rng, cap, n)
    gidx = gidx + base
    gidx[count:] = -1  # padding past the count, as a sharded sample leaves it
    gidx[: count // 10] = 7  # some foreign indices inside the prefix
    cnt = torch.tensor([count], dtype=torch.int64, device="cuda")
    d_idx = torch.from_numpy(gidx).cuda()  # kept alive until the kernel has run
    d_td = torch.from_numpy(td).cuda()
    rc = _lib.lib.per_update_priorities_shard_count(
        buf._store_ref, base, d_idx.data_ptr(), d_td.data_ptr(), n, cnt.data_ptr(),
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    assert rc == 0
    st = oracle.OracleStore(cap, {"x": 1})
    lv = np.zeros(st.capacity_padded, np.float32)
    lv[:cap] = leaves
    st.set_priorities(lv)
    own = gidx[:count] >= base
    st.update_priorities(gidx[:count][own] - base, td[:count][own])
    np.testing.assert_allclose(buf.priorities.cpu().numpy()[:cap], st.priorities[:cap],
                               rtol=1e-6, atol=0)
    check_tree(buf)
    s = buf.status()
    assert s["foreign"] == count // 10 and s["bad_indices"] == 0 and s["errors"] == 0


def _apply_and_check(cap, leaves, batches):
    buf = make_buffer(cap, {"x": 1}, None, leaves)
    st = oracle.OracleStore(cap, {"x": 1})
    lv = np.zeros(st.capacity_padded, np.float32)
    lv[:cap] = leaves
    st.set_priorities(lv)
    for idx, td in batches:
        buf.update_priorities(torch.from_numpy(idx).cuda(), torch.from_numpy(td).cuda())
        st.update_priorities(idx, td)
    np.testing.assert_allclose(buf.priorities.cpu().numpy()[:cap], st.priorities[:cap],
                               rtol=1e-6, atol=0)
    check_tree(buf)
    assert buf._max_priority.item() == pytest.approx(float(st.max_priority), rel=1e-6)
    s = buf.status()
    assert s["errors"] == 0 and s["timeouts"] == 0


def test_partitioned_update_one_top_node_many_rounds():
    """512 entries under one top-level node (one CTA takes them all: 16
    rounds of 32, duplicates across rounds): the last occurrence still wins;
    then 2048 such entries (64 rounds)."""
    rng = np.random.default_rng(5)
    cap = 1_000_000
    leaves = cases.leaves_abs_normal(rng, cap)
    node = 321  # top-level node of a 1M store: slots 321 * 1024 ...
    batches = []
    for m in (512, 2048):
        idx = (node * 1024 + rng.integers(0, 1024, m)).astype(np.int64)
        idx[rng.integers(0, m, 100)] = idx[rng.integers(0, m, 100)]  # more duplicates
        td = (rng.standard_normal(m) * 2).astype(np.float32)
        batches.append((idx, td))
    _apply_and_check(cap, leaves, batches)


def test_partitioned_update_one_slot_repeated():
    """Every entry names the same slot: the last TD error wins."""
    rng = np.random.default_rng(6)
    cap = 1_000_000
    leaves = cases.leaves_abs_normal(rng, cap)
    idx = np.full(300, 777_777, np.int64)
    td = rng.random(300).astype(np.float32)
    _apply_and_check(cap, leaves, [(idx, td)])
