"""TEST ONLY: a CPU shard with the semantics of the CUDA shard (numpy, oracle
arithmetic), so that ShardedPERBuffer's multi-rank host logic (all-gather of
shard totals, max all-reduce, update routing) can run on gloo ranks without a
GPU. The device kernels themselves are checked on the GPU."""

from __future__ import annotations

import numpy as np
import torch

from oracle import oracle


class CpuShard:
    def __init__(self, capacity, fields, alpha=0.6, eps=1e-6):
        self.st = oracle.OracleStore(capacity, fields, alpha=alpha, eps=eps)
        self.capacity = capacity
        self.device = torch.device("cpu")

    def add(self, batch):
        self.st.add({k: v.numpy() for k, v in batch.items()})

    def set_leaves(self, leaves):
        lv = np.zeros(self.st.capacity_padded, np.float32)
        lv[: leaves.size] = leaves
        self.st.set_priorities(lv)

    def stats(self, out):
        out[0] = float(np.sum(self.st.priorities[: self.capacity].astype(np.float64)))
        out[1] = float(self.st.size)

    def sample(self, rank, world, base, all_stats, rand, beta):
        stats = all_stats.numpy()
        totals, sizes = stats[:, 0], stats[:, 1]
        S = np.zeros(world + 1)
        for g in range(world):
            S[g + 1] = S[g] + totals[g]
        T32 = np.float32(S[world])
        N32 = np.float32(sizes.sum())
        r = rand.numpy().astype(np.float32)
        u = (r * T32).astype(np.float32)
        owner = np.searchsorted(S[1:], u.astype(np.float64), side="right")
        lastpos = max(g for g in range(world) if totals[g] > 0)
        owner = np.where(owner >= world, lastpos, owner)
        mine = np.nonzero(owner == rank)[0]
        p64 = np.cumsum(self.st.priorities[: self.capacity].astype(np.float64))
        t = u[mine].astype(np.float64) - S[rank]
        loc = np.minimum(np.searchsorted(p64, t, side="right"), self.st.size - 1)
        p = self.st.priorities[loc]
        w = np.power(N32 * (p / T32).astype(np.float32), np.float32(-beta)).astype(np.float32)
        b = r.size
        out = torch.zeros(b, self.st.row_dim)
        idx = torch.full((b,), -1, dtype=torch.int64)
        wt = torch.zeros(b)
        pos = torch.full((b,), -1, dtype=torch.int32)
        n = mine.size
        out[:n] = torch.from_numpy(self.st.storage[loc])
        idx[:n] = torch.from_numpy(loc + base)
        wt[:n] = torch.from_numpy(w)
        pos[:n] = torch.from_numpy(mine.astype(np.int32))
        lmax = torch.tensor([float(w.max()) if n else 0.0], dtype=torch.float32)
        return out, idx, wt, pos, torch.tensor([n], dtype=torch.int64), lmax

    def normalize(self, w, count, gmax):
        n = int(count.item())
        w[:n] = w[:n] / gmax

    def update(self, base, idx, td, count=None):
        if count is not None:  # only the owned prefix of a sharded sample's idx
            n = int(count.item())
            idx, td = idx[:n], td[:n]
        i = idx.numpy() - base
        keep = (i >= 0) & (i < self.capacity)
        if keep.any():
            self.st.update_priorities(i[keep], td.numpy()[keep])
