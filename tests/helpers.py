"""Shared helpers of the GPU parity tests: build a buffer from a seeded case
and compare its sample against the oracle (oracle/oracle.py)."""

from __future__ import annotations

import numpy as np
import torch

from oracle import oracle
from per_b200 import PERBuffer

# Tolerances of the parity contract: indices bit-exact except float32
# prefix-boundary ties (within 1 ulp of u, counted), gathered rows bit-exact,
# IS weights within 1e-6 relative, tree sums within 1e-5 relative of the
# exact sums of the leaves.
W_RTOL = 1e-6
SUM_RTOL = 1e-5


def make_buffer(capacity, fields, rows=None, leaves=None, alpha=0.6, eps=1e-6,
                storage_dtype=torch.float32):
    buf = PERBuffer(capacity, fields, device="cuda", alpha=alpha, eps=eps,
                    storage_dtype=storage_dtype)
    if rows is not None:
        buf.add({k: torch.as_tensor(v).cuda() for k, v in rows.items()})
    if leaves is not None:
        lv = np.zeros(buf.capacity_padded, np.float32)
        lv[: leaves.size] = leaves
        buf.priorities.copy_(torch.from_numpy(lv))
        buf.rebuild_sums()
    return buf


def packed_rows(rows, fields):
    return np.concatenate([np.asarray(rows[k], np.float32).reshape(len(rows[k]), -1)
                           for k in fields], axis=1)


def check_sample(buf, rows_np, leaves_np, size, rand_np, beta, golden_idx=None, tag=""):
    """Sample with the given uniforms and check it against the oracle.

    Returns a dict of counters (equal, excused ties)."""
    rand = torch.from_numpy(np.asarray(rand_np, np.float32)).cuda()
    views, idx, w = buf.sample_from_uniforms(rand, beta)
    out = torch.cat([views[k] for k in buf.fields], dim=1)
    torch.cuda.synchronize()
    idx_g = idx.cpu().numpy()
    w_g = w.cpu().numpy()
    out_g = out.cpu().numpy()

    cap = buf.capacity
    lv = np.zeros(buf.capacity_padded, np.float32)
    lv[: leaves_np.size] = leaves_np
    idx_o, w_o, csum = oracle.sample(lv, cap, size, rand_np, beta)
    ref_idx = idx_o if golden_idx is None else np.asarray(golden_idx)
    if golden_idx is not None:
        np.testing.assert_array_equal(idx_o, golden_idx)  # oracle still pinned
    eq, exc, bad = oracle.classify_indices(idx_g, ref_idx, rand_np, csum, size)
    assert bad.size == 0, (
        f"{tag}: {bad.size} index mismatches outside float32 ties, e.g. pos {bad[:5]} "
        f"gpu {idx_g[bad[:5]]} oracle {ref_idx[bad[:5]]}")
    assert (idx_g >= 0).all() and (idx_g < size).all()
    # rows: bit-exact copies of the stored rows
    np.testing.assert_array_equal(out_g, rows_np[idx_g])
    # weights: the oracle's formula on the engine's own indices
    w_ref = oracle.weights_for(lv, csum[-1], size, idx_g, beta)
    np.testing.assert_allclose(w_g, w_ref, rtol=W_RTOL, atol=0, err_msg=tag)
    if exc == 0:
        np.testing.assert_allclose(w_g, w_o, rtol=W_RTOL, atol=0, err_msg=tag)
    return {"equal": eq, "excused": exc, "n": idx_g.size}


def check_tree(buf, rtol=SUM_RTOL):
    """Every maintained sum level equals the exact sums of the leaves."""
    leaves = buf.priorities.cpu().numpy()
    for k in range(1, buf.num_levels):
        exact = oracle.tree_sums(leaves, buf.capacity, k)
        got = buf.level(k)[: exact.size].cpu().numpy().astype(np.float64)
        np.testing.assert_allclose(got, exact, rtol=rtol, atol=1e-30, err_msg=f"level {k}")
