"""Seeded inputs of the golden cases (numpy only, no reference import).

Each case is a deterministic function of its seed, so a machine without the
reference rebuilds the same inputs that make_golden.py fed to the reference; every case also
carries a SHA-256 of its inputs, stored in the fixture, to catch any drift.
Shapes and value distributions follow the workloads the reference is measured
on (config 1 of the CPU run: capacity 100,000, fields obs32/action8/reward1/
next_obs32/done1 = row_dim 74, priorities (|N(0,1)|+1e-6)^0.6, batch 256,
beta 0.4, then 256 |N(0,1)| TD errors with ~10% duplicate indices).
"""

from __future__ import annotations

import hashlib

import numpy as np

FIELDS_74 = {"obs": 32, "action": 8, "reward": 1, "next_obs": 32, "done": 1}


def digest(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        a = np.ascontiguousarray(a)
        h.update(str(a.dtype).encode())
        h.update(str(a.shape).encode())
        h.update(a.tobytes())
    return h.hexdigest()


def rows_74(rng, n):
    rows = {
        "obs": rng.standard_normal((n, 32), dtype=np.float32),
        "action": rng.standard_normal((n, 8), dtype=np.float32),
        "reward": rng.standard_normal((n, 1), dtype=np.float32),
        "next_obs": rng.standard_normal((n, 32), dtype=np.float32),
        "done": (rng.random((n, 1)) < 0.5).astype(np.float32),
    }
    return rows


def leaves_abs_normal(rng, n, alpha=0.6, eps=1e-6):
    x = np.abs(rng.standard_normal(n)).astype(np.float32)
    return np.power(x + np.float32(eps), np.float32(alpha)).astype(np.float32)


def dup_indices(rng, idx, frac):
    """Replace ~frac of the entries by copies of other entries of the batch."""
    idx = np.array(idx, np.int64)
    n = idx.size
    k = max(1, int(round(frac * n)))
    pos = rng.choice(n, size=k, replace=False)
    src = rng.integers(0, n, size=k)
    idx[pos] = idx[src]
    return idx


def case_config1(seed=1):
    """CPU config: cap 100,000 x 74, sample 256 beta 0.4, update 256 with ~10% dups."""
    rng = np.random.default_rng(seed)
    cap = 100_000
    rows = rows_74(rng, cap)
    leaves = leaves_abs_normal(rng, cap)
    rand = rng.random(256, dtype=np.float32)
    td = np.abs(rng.standard_normal(256)).astype(np.float32)
    rand2 = rng.random(256, dtype=np.float32)
    dup = np.random.default_rng(seed + 1000)
    return dict(capacity=cap, fields=FIELDS_74, rows=rows, leaves=leaves, size=cap,
                rand=rand, beta=0.4, td=td, rand2=rand2, dup_rng=dup, dup_frac=0.10)


def case_small(seed=2):
    """cap 5000 (last block half padding), full, row_dim 3."""
    rng = np.random.default_rng(seed)
    cap = 5000
    rows = {"x": rng.standard_normal((cap, 3), dtype=np.float32)}
    leaves = leaves_abs_normal(rng, cap)
    rand = rng.random(4096, dtype=np.float32)
    return dict(capacity=cap, fields={"x": 3}, rows=rows, leaves=leaves, size=cap,
                rand=rand, beta=0.4)


def case_partial(seed=3):
    """cap 4096, only 3000 live slots (size < capacity)."""
    rng = np.random.default_rng(seed)
    cap, size = 4096, 3000
    rows = {"x": rng.standard_normal((size, 2), dtype=np.float32)}
    leaves = np.zeros(cap, np.float32)
    leaves[:size] = leaves_abs_normal(rng, size)
    rand = rng.random(4096, dtype=np.float32)
    return dict(capacity=cap, fields={"x": 2}, rows=rows, leaves=leaves, size=size,
                rand=rand, beta=0.7)


def case_ties(seed=4):
    """Leaves on a coarse dyadic grid so u = rand*total often hits a prefix exactly."""
    rng = np.random.default_rng(seed)
    cap = 3000
    rows = {"x": np.arange(cap, dtype=np.float32).reshape(cap, 1)}
    leaves = (rng.integers(1, 8, cap).astype(np.float32) * np.float32(0.25))
    # rand values that land exactly on prefix boundaries
    csum = np.cumsum(leaves.astype(np.float64)).astype(np.float32)
    total = csum[-1]
    pick = rng.integers(0, cap - 1, 2048)
    rand = (csum[pick] / total).astype(np.float32)
    rand = np.concatenate([rand, rng.random(2048, dtype=np.float32)])
    return dict(capacity=cap, fields={"x": 1}, rows=rows, leaves=leaves, size=cap,
                rand=rand, beta=0.5)


def case_heavy(seed=5):
    """lognormal(0,2) priorities with 1% exact zeros (batch-sweep distribution)."""
    rng = np.random.default_rng(seed)
    cap = 20_000
    rows = {"x": rng.standard_normal((cap, 4), dtype=np.float32)}
    leaves = rng.lognormal(0.0, 2.0, cap).astype(np.float32)
    zeros = rng.choice(cap, cap // 100, replace=False)
    leaves[zeros] = 0.0
    leaves[cap - 1] = 1.0  # keep the clamp slot positive so the oracle stays finite
    rand = rng.random(8192, dtype=np.float32)
    return dict(capacity=cap, fields={"x": 4}, rows=rows, leaves=leaves, size=cap,
                rand=rand, beta=0.4)


def case_update_dups(seed=6):
    """cap 2048: updates with heavy duplicates, divergent values, all-same index."""
    rng = np.random.default_rng(seed)
    cap = 2048
    leaves = leaves_abs_normal(rng, cap)
    idx = np.concatenate([np.full(64, 7), np.full(64, 700), rng.integers(0, cap, 512),
                          np.zeros(32, np.int64)]).astype(np.int64)
    td = np.concatenate([np.linspace(0.5, 5.0, 64), np.linspace(1.0, 9.0, 64),
                         rng.standard_normal(512) * 3, np.linspace(0.1, 5, 32)]).astype(np.float32)
    return dict(capacity=cap, leaves=leaves, idx=idx, td=td, alpha=0.6, eps=1e-6)


def case_update_storm(seed=7):
    """cap 30,000: 16,384 indices, 50% of them repeating an index of the other half."""
    rng = np.random.default_rng(seed)
    cap = 30_000
    leaves = leaves_abs_normal(rng, cap)
    half = rng.integers(0, cap, 8192)
    rep = half[rng.integers(0, 8192, 8192)]
    idx = np.concatenate([half, rep])
    rng.shuffle(idx)
    td = np.abs(rng.standard_normal(idx.size)).astype(np.float32) * 2
    return dict(capacity=cap, leaves=leaves, idx=idx.astype(np.int64), td=td,
                alpha=0.6, eps=1e-6)


def case_add_wrap(seed=8):
    """cap 1000: add 750, update, add 750 (wraps 1.5 laps), add 2500 (> capacity)."""
    rng = np.random.default_rng(seed)
    cap = 1000
    adds = [rng.standard_normal((750, 3), dtype=np.float32),
            rng.standard_normal((750, 3), dtype=np.float32),
            rng.standard_normal((2500, 3), dtype=np.float32)]
    upd_idx = rng.integers(0, 750, 300).astype(np.int64)
    upd_td = (np.abs(rng.standard_normal(300)) * 7).astype(np.float32)
    return dict(capacity=cap, fields={"x": 3}, adds=adds, upd_idx=upd_idx, upd_td=upd_td)


def case_sumtree(seed=12):
    """The reference's CPU sum tree (baselines/cpu_sumtree.py) on cap 1000 (not a
    power of two): add 700, update 300 with duplicates, sample 512; add 500
    (wraps), update 400 with larger TD errors, sample 512."""
    rng = np.random.default_rng(seed)
    cap = 1000
    adds = [rng.standard_normal((700, 3), dtype=np.float32),
            rng.standard_normal((500, 3), dtype=np.float32)]
    upd_idx = [dup_indices(rng, rng.integers(0, 700, 300), 0.1),
               dup_indices(rng, rng.integers(0, cap, 400), 0.1)]
    upd_td = [np.abs(rng.standard_normal(300)).astype(np.float32),
              (np.abs(rng.standard_normal(400)) * 5).astype(np.float32)]
    rand = [rng.random(512), rng.random(512)]
    return dict(capacity=cap, fields={"x": 3}, adds=adds, upd_idx=upd_idx, upd_td=upd_td,
                rand=rand, beta=0.4)


def sumtree_inputs_digest(c) -> str:
    return digest(*c["adds"], *c["upd_idx"], *c["upd_td"], *c["rand"])


SAMPLE_CASES = {
    "config1": case_config1,
    "small": case_small,
    "partial": case_partial,
    "ties": case_ties,
    "heavy": case_heavy,
}


def sample_inputs_digest(c) -> str:
    parts = [c["leaves"], c["rand"]] + [c["rows"][k] for k in sorted(c["rows"])]
    return digest(*parts)
