"""Prioritized replay buffer sharded over the ranks of a process group.

No counterpart in triton-per (which has no multi-GPU code); it keeps the
single-buffer semantics of `PERBuffer` (src/triton_per/buffer.py:82-105,
:133-145) over a capacity split across GPUs, one process per GPU.

Rank g owns the global slots [g * C, (g + 1) * C) with C = ceil(capacity /
world), in its own store on its own GPU; rows never leave their GPU.

sample(batch_size, beta) is collective. Every rank draws the same
`batch_size` global uniforms (a generator seeded identically on every rank),
and the ranks exchange their shard totals and sizes (all-gather of 16 bytes
per rank). A draw u = rand * total belongs to the shard whose range of the
global priority prefix holds u: the union of the ranks' draws is exactly the
draw of one buffer holding every slot, with IS weights (N * p / total)^-beta
over the global size N and total. Each rank returns the draws it owns,
compacted into the first `count` entries of full-size outputs (count is a
device tensor; positions in the global batch are in `pos`); the weights are
normalised by the max over all ranks (all-reduce of one float).

update_priorities(idx, td) applies the entries whose global index this rank
owns (the data-parallel case: every rank updates the draws it sampled); with
route=True every rank's entries are all-gathered first, so a rank may update
slots sampled elsewhere.

add(batch) is rank-local: each rank inserts its own transitions.
"""

from __future__ import annotations

import ctypes
import math
from typing import NamedTuple

import torch
import torch.distributed as dist

from . import _lib
from .buffer import PERBuffer, _stream_ptr


class ShardSample(NamedTuple):
    views: dict          # field name -> [batch_size, d] views; first `count` rows valid
    idx: torch.Tensor    # int64[batch_size] global slot indices (first `count` valid)
    w: torch.Tensor      # float32[batch_size] normalised IS weights (first `count` valid)
    count: torch.Tensor  # int64[1] device: draws owned by this rank
    pos: torch.Tensor    # int32[batch_size] positions of those draws in the global batch


class CudaShard:
    """The rank's shard on its GPU: a PERBuffer driven through the C ABI."""

    def __init__(self, capacity, fields, device, alpha, eps):
        self.buf = PERBuffer(capacity, fields, device=device, alpha=alpha, eps=eps)
        self.device = self.buf.device

    def add(self, batch):
        self.buf.add(batch)

    def stats(self, out: torch.Tensor) -> None:
        with torch.cuda.device(self.device):
            _lib.check("per_shard_stats", _lib.lib.per_shard_stats(
                self.buf._store_ref, out.data_ptr(), _stream_ptr(self.device)))

    def sample(self, rank, world, base, all_stats, rand, beta):
        b = rand.numel()
        dev = self.device
        out = torch.empty(b, self.buf.row_dim, device=dev)
        idx = torch.empty(b, dtype=torch.int64, device=dev)
        w = torch.empty(b, device=dev)
        pos = torch.empty(b, dtype=torch.int32, device=dev)
        count = torch.empty(1, dtype=torch.int64, device=dev)
        lmax = torch.empty(1, device=dev)
        with torch.cuda.device(dev):
            _lib.check("per_sample_sharded", _lib.lib.per_sample_sharded(
                self.buf._store_ref, rank, world, base, all_stats.data_ptr(), rand.data_ptr(), b,
                float(beta), out.data_ptr(), self.buf.row_dim, idx.data_ptr(), w.data_ptr(),
                pos.data_ptr(), count.data_ptr(), lmax.data_ptr(), _stream_ptr(dev)))
        return out, idx, w, pos, count, lmax

    def normalize(self, w, count, gmax):
        with torch.cuda.device(self.device):
            _lib.check("per_normalize", _lib.lib.per_normalize(
                w.data_ptr(), count.data_ptr(), gmax.data_ptr(), w.numel(),
                _stream_ptr(self.device)))

    def update(self, base, idx, td):
        with torch.cuda.device(self.device):
            _lib.check("per_update_priorities_shard", _lib.lib.per_update_priorities_shard(
                self.buf._store_ref, base, idx.data_ptr(), td.data_ptr(), idx.numel(),
                _stream_ptr(self.device)))


class ShardedPERBuffer:
    def __init__(
        self,
        capacity: int,
        fields: dict[str, int],
        device: str | torch.device = "cuda",
        alpha: float = 0.6,
        eps: float = 1e-6,
        group=None,
        seed: int = 0,
        shard=None,
    ):
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.capacity = capacity
        self.fields = dict(fields)
        self.alpha = alpha
        self.eps = eps
        self.shard_capacity = -(-capacity // self.world)
        self.base = self.rank * self.shard_capacity
        self.shard = shard if shard is not None else CudaShard(
            self.shard_capacity, fields, torch.device(device), alpha, eps)
        self.device = self.shard.device
        self.row_dim = sum(fields.values())
        self._offsets = {}
        o = 0
        for name, d in fields.items():
            self._offsets[name] = (o, o + d)
            o += d
        # identical uniform streams on every rank
        self._gen = torch.Generator(device=self.device).manual_seed(seed)
        self._stats = torch.zeros(2, dtype=torch.float64, device=self.device)
        self._all_flat = torch.zeros(self.world * 2, dtype=torch.float64, device=self.device)
        self._all_stats = self._all_flat.view(self.world, 2)

    # ------------------------------------------------------------------ add
    def add(self, batch: dict[str, torch.Tensor]) -> None:
        """Insert this rank's transitions into its own shard."""
        self.shard.add(batch)

    # --------------------------------------------------------------- sample
    def sample(self, batch_size: int, beta: float = 0.4) -> ShardSample:
        """Collective: this rank's share of a global batch of `batch_size` draws."""
        rand = torch.rand(batch_size, generator=self._gen, device=self.device)
        return self.sample_from_uniforms(rand, beta)

    def sample_from_uniforms(self, rand: torch.Tensor, beta: float = 0.4) -> ShardSample:
        """sample() with caller-provided global uniforms (identical on every rank)."""
        rand = rand.to(device=self.device, dtype=torch.float32).contiguous()
        self.shard.stats(self._stats)
        dist.all_gather_into_tensor(self._all_flat, self._stats, group=self.group)
        out, idx, w, pos, count, lmax = self.shard.sample(
            self.rank, self.world, self.base, self._all_stats, rand, beta)
        dist.all_reduce(lmax, op=dist.ReduceOp.MAX, group=self.group)
        self.shard.normalize(w, count, lmax)
        views = {name: out[:, a:b] for name, (a, b) in self._offsets.items()}
        return ShardSample(views, idx, w, count, pos)

    # --------------------------------------------------------------- update
    def update_priorities(self, indices: torch.Tensor, td_errors: torch.Tensor,
                          route: bool = False) -> None:
        """Apply the entries this rank owns (global indices; -1 = padding).

        route=True all-gathers every rank's entries first (same length on
        every rank), so that TD errors computed on one rank reach the owner."""
        idx = indices.reshape(-1).to(device=self.device, dtype=torch.int64).contiguous()
        td = td_errors.detach().reshape(-1).to(device=self.device, dtype=torch.float32).contiguous()
        if idx.numel() != td.numel():
            raise ValueError(f"{idx.numel()} indices but {td.numel()} TD errors")
        if route and self.world > 1:
            all_idx = torch.empty(self.world * idx.numel(), dtype=torch.int64, device=self.device)
            all_td = torch.empty(self.world * td.numel(), dtype=torch.float32, device=self.device)
            dist.all_gather_into_tensor(all_idx, idx, group=self.group)
            dist.all_gather_into_tensor(all_td, td, group=self.group)
            idx, td = all_idx, all_td
        self.shard.update(self.base, idx, td)

    def global_stats(self) -> torch.Tensor:
        """[world, 2] (total priority, live size) of every shard (collective)."""
        self.shard.stats(self._stats)
        dist.all_gather_into_tensor(self._all_flat, self._stats, group=self.group)
        return self._all_stats.clone()
