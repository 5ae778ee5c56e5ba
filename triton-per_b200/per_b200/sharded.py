"""Prioritized replay buffer sharded over the ranks of a process group.

No counterpart in triton-per (which has no multi-GPU code); it keeps the
single-buffer semantics of `PERBuffer` (src/triton_per/buffer.py:82-105,
:133-145) over a capacity split across GPUs, one process per GPU.

Rank g owns the global slots [g * C, (g + 1) * C) with C = ceil(capacity /
world), in its own store on its own GPU; rows never leave their GPU.

sample(batch_size, beta) is collective. Every rank draws the same
`batch_size` global uniforms (a Philox stream drawn inside the sample
kernel, with the same seed and position on every rank),
and the ranks exchange their shard totals and sizes (16 bytes per rank). A
draw u = rand * total belongs to the shard whose range of the global priority
prefix holds u: the union of the ranks' draws is exactly the draw of one
buffer holding every slot, with IS weights (N * p / total)^-beta over the
global size N and total. Each rank returns the draws it owns, compacted into
the first `count` entries of full-size outputs (count is a device tensor;
positions in the global batch are in `pos`); the weights are normalised by
the max over all ranks.

The two exchanges run one of two ways:
- peer memory (`exchange="p2p"`, the default when every rank has a GPU of
  its own on one host): one kernel per sample; the statistics and the max
  weight cross NVLink as system-scope stores into CUDA-IPC-mapped mailboxes,
  waited on inside the kernel (bounded waits). Batches up to one wave of the
  kernel (`p2p_max_batch`, ~75k draws on a B200);
- collectives (`exchange="nccl"`, and larger batches): stats kernel,
  all-gather, sample kernel, all-reduce MAX, normalise kernel.

normalize="rank" normalises each rank's weights by the largest weight among
the draws that rank owns (a per-rank constant factor on the global-max
weights; the draws, rows and relative weights are unchanged). It leaves out
the max exchange, so the in-kernel path crosses NVLink once per sample
instead of twice, and the collective path skips its all-reduce. The default,
normalize="global", keeps the single-buffer weights exactly.

update_priorities(idx, td) applies the entries whose global index this rank
owns (the data-parallel case: every rank updates the draws it sampled); with
route=True every rank's entries are all-gathered first, so a rank may update
slots sampled elsewhere.

add(batch) is rank-local: each rank inserts its own transitions.
"""

from __future__ import annotations

import ctypes
import math
import os
import socket
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


class ShardSampleOut:
    """Caller-owned destination of one sharded sample (device tensors of the
    global batch size): rows with per-field views, idx (with the owned count
    stored right behind it), w and pos. Made by ShardedPERBuffer.sample_out();
    sample(..., out=) then allocates nothing."""

    def __init__(self, owner: "ShardedPERBuffer", batch: int, rows=None):
        if batch < 1:
            raise ValueError("batch must be positive")
        dev = owner.device
        if rows is None:
            rows = torch.empty(batch, owner.row_dim, device=dev)
        if rows.device != dev or rows.dtype != torch.float32 or \
                tuple(rows.shape) != (batch, owner.row_dim) or rows.stride(1) != 1:
            raise ValueError(f"rows must be [{batch}, {owner.row_dim}] float32 on {dev} "
                             "with unit column stride")
        self.owner = owner
        self.batch = batch
        self.rows = rows
        self._idx_count = torch.empty(batch + 1, dtype=torch.int64, device=dev)
        self.idx = self._idx_count[:batch]
        self.count = self._idx_count[batch:]
        self.w = torch.empty(batch, device=dev)
        self.pos = torch.empty(batch, dtype=torch.int32, device=dev)
        self.views = owner._views(rows)


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

    def sample(self, rank, world, base, all_stats, rand, beta, rng=None, batch=None):
        """rand: global uniforms; or rng = (seed, device int64 counter) and `batch`."""
        b = rand.numel() if rng is None else batch
        dev = self.device
        out = torch.empty(b, self.buf.row_dim, device=dev)
        idx = torch.empty(b, dtype=torch.int64, device=dev)
        w = torch.empty(b, device=dev)
        pos = torch.empty(b, dtype=torch.int32, device=dev)
        count = torch.empty(1, dtype=torch.int64, device=dev)
        lmax = torch.empty(1, device=dev)
        with torch.cuda.device(dev):
            if rng is None:
                _lib.check("per_sample_sharded", _lib.lib.per_sample_sharded(
                    self.buf._store_ref, rank, world, base, all_stats.data_ptr(), rand.data_ptr(),
                    b, float(beta), out.data_ptr(), self.buf.row_dim, idx.data_ptr(),
                    w.data_ptr(), pos.data_ptr(), count.data_ptr(), lmax.data_ptr(),
                    _stream_ptr(dev)))
            else:
                _lib.check("per_sample_sharded_rng", _lib.lib.per_sample_sharded_rng(
                    self.buf._store_ref, rank, world, base, all_stats.data_ptr(), rng[0],
                    rng[1].data_ptr(), b, float(beta), out.data_ptr(), self.buf.row_dim,
                    idx.data_ptr(), w.data_ptr(), pos.data_ptr(), count.data_ptr(),
                    lmax.data_ptr(), _stream_ptr(dev)))
        return out, idx, w, pos, count, lmax

    def sample_p2p_into(self, rank, world, base, mailboxes, beta, rng, out: ShardSampleOut,
                        local: bool = False):
        """sample_p2p with in-kernel uniforms into a caller-owned destination."""
        buf = self.buf
        args = (rank, world, base, mailboxes.data_ptr(), out.batch, float(beta), rng[0],
                rng[1].data_ptr(), out.rows.data_ptr(), out.rows.stride(0), out.idx.data_ptr(),
                out.w.data_ptr(), out.pos.data_ptr(), out.count.data_ptr())
        name = "per_sample_sharded_p2p_local_rng" if local else "per_sample_sharded_p2p_rng"
        if buf._engine is not None:
            rc = buf._engine.sample_sharded_p2p_into(*args, bool(local))
            if rc:
                _lib.check(name, rc)
        else:
            buf._call(name, getattr(_lib.lib, name),
                      buf._store_ref, args[0], args[1], args[2], args[3], args[6], args[7],
                      args[4], args[5], args[8], args[9], args[10], args[11], args[12], args[13])

    def sample_p2p(self, rank, world, base, mailboxes, rand, beta, rng=None, batch=None,
                   local: bool = False):
        """local (in-kernel uniforms only): weights normalised by this rank's max."""
        b = rand.numel() if rng is None else batch
        buf = self.buf
        if local and rng is None:
            raise ValueError("rank-local normalisation needs the in-kernel uniforms")
        if rng is not None and buf._engine is not None:
            rc, views, idx, w, pos, count = buf._engine.sample_sharded_p2p(
                rank, world, base, mailboxes.data_ptr(), b, float(beta), rng[0],
                rng[1].data_ptr(), bool(local))
            if rc:
                _lib.check("per_sample_sharded_p2p_rng", rc)
            return views, idx, w, pos, count
        dev = self.device
        out, idx_count, w = buf._outputs(b, extra_idx=1)
        idx, count = idx_count[:b], idx_count[b:]
        pos = torch.empty(b, dtype=torch.int32, device=dev)
        if rng is None:
            buf._call("per_sample_sharded_p2p", _lib.lib.per_sample_sharded_p2p, buf._store_ref,
                      rank, world, base, mailboxes.data_ptr(), rand.data_ptr(), b, float(beta),
                      out.data_ptr(), buf.row_dim, idx.data_ptr(), w.data_ptr(), pos.data_ptr(),
                      count.data_ptr())
        else:
            name = "per_sample_sharded_p2p_local_rng" if local else "per_sample_sharded_p2p_rng"
            buf._call(name, getattr(_lib.lib, name),
                      buf._store_ref, rank, world, base, mailboxes.data_ptr(), rng[0],
                      rng[1].data_ptr(), b, float(beta), out.data_ptr(), buf.row_dim,
                      idx.data_ptr(), w.data_ptr(), pos.data_ptr(), count.data_ptr())
        return out, idx, w, pos, count

    def p2p_max_batch(self) -> int:
        m = ctypes.c_int64(0)
        with torch.cuda.device(self.device):
            _lib.check("per_sample_sharded_p2p_max_batch",
                       _lib.lib.per_sample_sharded_p2p_max_batch(self.buf._store_ref, ctypes.byref(m)))
        return int(m.value)

    def normalize(self, w, count, gmax):
        with torch.cuda.device(self.device):
            _lib.check("per_normalize", _lib.lib.per_normalize(
                w.data_ptr(), count.data_ptr(), gmax.data_ptr(), w.numel(),
                _stream_ptr(self.device)))

    def update(self, base, idx, td, count=None):
        if count is None:
            self.buf._call("per_update_priorities_shard", _lib.lib.per_update_priorities_shard,
                           self.buf._store_ref, base, idx.data_ptr(), td.data_ptr(), idx.numel())
        elif self.buf._engine is not None:  # only the first *count entries
            rc = self.buf._engine.update_shard_count(base, idx, td, count)
            if rc:
                _lib.check("per_update_priorities_shard_count", rc)
        else:  # only the first *count entries (a sharded sample's owned draws)
            self.buf._call("per_update_priorities_shard_count",
                           _lib.lib.per_update_priorities_shard_count, self.buf._store_ref, base,
                           idx.data_ptr(), td.data_ptr(), idx.numel(), count.data_ptr())


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
        exchange: str = "auto",
        normalize: str = "global",
    ):
        if exchange not in ("auto", "p2p", "nccl"):
            raise ValueError(f"exchange must be 'auto', 'p2p' or 'nccl', not {exchange!r}")
        if normalize not in ("global", "rank"):
            raise ValueError(f"normalize must be 'global' or 'rank', not {normalize!r}")
        self.normalize = normalize
        self.group = group
        distributed = dist.is_available() and dist.is_initialized()
        self.rank = dist.get_rank(group) if distributed else 0
        self.world = dist.get_world_size(group) if distributed else 1
        self.capacity = capacity
        self.fields = dict(fields)
        self.alpha = alpha
        self.eps = eps
        if self.world > 1:  # every rank must build the same buffer (checked collectively)
            mine = (int(capacity), tuple(self.fields.items()), float(alpha), float(eps), int(seed))
            everyone = [None] * self.world
            dist.all_gather_object(everyone, mine, group=group)
            if any(o != everyone[0] for o in everyone):
                raise ValueError("ShardedPERBuffer: ranks disagree on capacity, fields, alpha, eps "
                                 f"or seed: {everyone}")
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
        self._names = tuple(self._offsets)
        self._dims = tuple(b - a for a, b in self._offsets.values())
        # identical uniform streams on every rank: the in-kernel Philox stream
        # (seed, device counter) of the CUDA shard; a torch generator for
        # other shard types
        self.seed = int(seed) & 0xFFFFFFFFFFFFFFFF
        self._gen = torch.Generator(device=self.device).manual_seed(seed)
        self._rng_counter = torch.zeros(1, dtype=torch.int64, device=self.device)
        self._stats = torch.zeros(2, dtype=torch.float64, device=self.device)
        self._all_flat = torch.zeros(self.world * 2, dtype=torch.float64, device=self.device)
        self._all_stats = self._all_flat.view(self.world, 2)
        self._last = None          # (idx, count) of the last sample on this rank
        self._mailbox = None       # own mailbox (device pointer)
        self._peer_boxes = []      # peers' mailboxes mapped into this process
        self._mailboxes = None     # int64[world] device array of mailbox pointers
        self.p2p_max_batch = 0
        self.exchange = "nccl"
        if exchange != "nccl" and isinstance(self.shard, CudaShard):
            self._setup_p2p(required=exchange == "p2p")

    # ------------------------------------------------------------ p2p set-up
    def _p2p_possible(self) -> bool:
        """Every rank on its own GPU of one host (the kernels wait on one another)."""
        if self.world == 1:
            return True
        try:
            gpu = str(torch.cuda.get_device_properties(self.device).uuid)
        except (AttributeError, RuntimeError):
            gpu = f"{os.environ.get('CUDA_VISIBLE_DEVICES', '')}:{self.device.index}"
        me = (socket.gethostname(), gpu)
        everyone = [None] * self.world
        dist.all_gather_object(everyone, me, group=self.group)
        return len({h for h, _ in everyone}) == 1 and len({u for _, u in everyone}) == self.world

    def _setup_p2p(self, required: bool) -> None:
        if self.world > 1 and dist.get_backend(self.group) != "nccl":  # same on every rank
            if required:
                raise RuntimeError("exchange='p2p' needs the nccl backend")
            return
        ok = self._p2p_possible()
        if ok:
            box = ctypes.c_void_p()
            handle = (ctypes.c_char * _lib.IPC_HANDLE_BYTES)()
            with torch.cuda.device(self.device):
                rc = _lib.lib.per_mailbox_create(ctypes.byref(box), handle)
            ok = rc == 0
            if ok:
                self._mailbox = box.value
        if self.world > 1:  # every rank takes the same path
            flag = torch.tensor([1.0 if ok else 0.0], device=self.device)
            dist.all_reduce(flag, op=dist.ReduceOp.MIN, group=self.group)
            ok = flag.item() == 1.0
        if ok:
            handles = [bytes(handle)] * self.world
            if self.world > 1:
                dist.all_gather_object(handles, bytes(handle), group=self.group)
            ptrs = []
            opened = True
            for g in range(self.world):
                if g == self.rank:
                    ptrs.append(self._mailbox)
                    continue
                p = ctypes.c_void_p()
                with torch.cuda.device(self.device):
                    rc = _lib.lib.per_mailbox_open(handles[g], ctypes.byref(p))
                if rc:
                    opened = False
                    break
                self._peer_boxes.append(p.value)
                ptrs.append(p.value)
            mb = self.shard.p2p_max_batch() if opened else 0
            if self.world > 1:
                t = torch.tensor([float(opened), float(mb)], device=self.device)
                t_all = torch.empty(self.world * 2, device=self.device)
                dist.all_gather_into_tensor(t_all, t, group=self.group)
                t_all = t_all.view(self.world, 2)
                opened = bool(t_all[:, 0].min().item() == 1.0)
                mb = int(t_all[:, 1].min().item())
            if opened:
                self._mailboxes = torch.tensor(ptrs, dtype=torch.int64, device=self.device)
                self.p2p_max_batch = mb
                self.exchange = "p2p"
                if self.world > 1:
                    dist.barrier(group=self.group)
                return
            self._release_mailboxes()
        if required:
            raise RuntimeError("exchange='p2p' needs one GPU per rank on one host and CUDA IPC")

    def _release_mailboxes(self) -> None:
        with torch.cuda.device(self.device):
            for p in self._peer_boxes:
                _lib.lib.per_mailbox_close(ctypes.c_void_p(p))
            self._peer_boxes = []
            if self._mailbox is not None:
                _lib.lib.per_mailbox_destroy(ctypes.c_void_p(self._mailbox))
                self._mailbox = None
        self._mailboxes = None
        self.p2p_max_batch = 0
        self.exchange = "nccl"

    def close(self) -> None:
        """Collective: unmap and free the mailboxes (peer-memory exchange)."""
        if self._mailbox is None:
            return
        torch.cuda.synchronize(self.device)
        if self.world > 1:
            dist.barrier(group=self.group)  # no peer still writes into our mailbox
        self._release_mailboxes()

    # ------------------------------------------------------------------ add
    def add(self, batch: dict[str, torch.Tensor]) -> None:
        """Insert this rank's transitions into its own shard."""
        self.shard.add(batch)

    # --------------------------------------------------------------- sample
    def sample_out(self, batch_size: int, rows: torch.Tensor | None = None) -> ShardSampleOut:
        """A reusable destination for sample(batch_size, beta, out=...); `rows`
        may be a view into the caller's own buffer (e.g. one slot of a
        [rounds, batch, row_dim] block that goes to the host in one copy)."""
        return ShardSampleOut(self, int(batch_size), rows)

    def sample(self, batch_size: int, beta: float = 0.4,
               out: ShardSampleOut | None = None) -> ShardSample:
        """Collective: this rank's share of a global batch of `batch_size` draws.

        With `out` (from sample_out(); in-kernel exchange only, batch up to
        p2p_max_batch) the draws are written into that destination and nothing
        is allocated."""
        if out is not None:
            if out.owner is not self or out.batch != int(batch_size):
                raise ValueError("out was made by sample_out() of another buffer or batch size")
            if self.exchange != "p2p" or out.batch > self.p2p_max_batch:
                raise ValueError("sample(out=) needs the in-kernel exchange and a batch of at "
                                 f"most p2p_max_batch ({self.p2p_max_batch})")
            self.shard.sample_p2p_into(self.rank, self.world, self.base, self._mailboxes, beta,
                                       (self.seed, self._rng_counter), out,
                                       local=self.normalize == "rank")
            self._last = (out.idx, out.count)
            return ShardSample(out.views, out.idx, out.w, out.count, out.pos)
        if not isinstance(self.shard, CudaShard):
            rand = torch.rand(batch_size, generator=self._gen, device=self.device)
            return self.sample_from_uniforms(rand, beta)
        rng = (self.seed, self._rng_counter)
        if self.exchange == "p2p" and batch_size <= self.p2p_max_batch:
            out, idx, w, pos, count = self.shard.sample_p2p(
                self.rank, self.world, self.base, self._mailboxes, None, beta, rng, batch_size,
                local=self.normalize == "rank")
            self._last = (idx, count)
            views = out if isinstance(out, dict) else self._views(out)
            return ShardSample(views, idx, w, count, pos)
        else:
            self._exchange_stats()
            out, idx, w, pos, count, lmax = self.shard.sample(
                self.rank, self.world, self.base, self._all_stats, None, beta, rng, batch_size)
            if self.world > 1 and self.normalize == "global":
                dist.all_reduce(lmax, op=dist.ReduceOp.MAX, group=self.group)
            self.shard.normalize(w, count, lmax)
        self._last = (idx, count)
        return ShardSample(self._views(out), idx, w, count, pos)

    def _views(self, out):
        return dict(zip(self._names, out.split(self._dims, dim=1)))

    def sample_from_uniforms(self, rand: torch.Tensor, beta: float = 0.4) -> ShardSample:
        """sample() with caller-provided global uniforms (identical on every rank)."""
        rand = rand.to(device=self.device, dtype=torch.float32).contiguous()
        if self.exchange == "p2p" and rand.numel() <= self.p2p_max_batch and \
                self.normalize == "global":
            out, idx, w, pos, count = self.shard.sample_p2p(
                self.rank, self.world, self.base, self._mailboxes, rand, beta)
            views = {name: out[:, a:b] for name, (a, b) in self._offsets.items()}
            return ShardSample(views, idx, w, count, pos)
        self._exchange_stats()
        out, idx, w, pos, count, lmax = self.shard.sample(
            self.rank, self.world, self.base, self._all_stats, rand, beta)
        if self.world > 1 and self.normalize == "global":
            dist.all_reduce(lmax, op=dist.ReduceOp.MAX, group=self.group)
        self.shard.normalize(w, count, lmax)
        views = {name: out[:, a:b] for name, (a, b) in self._offsets.items()}
        return ShardSample(views, idx, w, count, pos)

    # --------------------------------------------------------------- update
    def update_priorities(self, indices: torch.Tensor, td_errors: torch.Tensor,
                          route: bool = False) -> None:
        """Apply the entries this rank owns (global indices; -1 = padding).

        route=True all-gathers every rank's entries first (same length on
        every rank), so that TD errors computed on one rank reach the owner.
        When `indices` is the idx tensor of this rank's last sample, only its
        owned prefix (the sample's device count) is read."""
        count = None
        if not route and self._last is not None and indices is self._last[0]:
            count = self._last[1]
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
        if count is None:
            self.shard.update(self.base, idx, td)
        else:
            self.shard.update(self.base, idx, td, count)

    def state_dict(self) -> dict:
        """This rank's shard (PERBuffer.state_dict) plus the sharding and the
        shared uniform-stream position; each rank saves its own."""
        if not isinstance(self.shard, CudaShard):
            raise TypeError("state_dict needs the CUDA shard")
        return {"rank": self.rank, "world": self.world, "capacity": self.capacity,
                "seed": self.seed, "rng_counter": int(self._rng_counter.item()),
                "shard": self.shard.buf.state_dict()}

    def load_state_dict(self, state: dict) -> None:
        if state["world"] != self.world or state["rank"] != self.rank or \
                state["capacity"] != self.capacity:
            raise ValueError("sharded state was saved by another rank or layout")
        self.seed = int(state["seed"])
        self._rng_counter.fill_(int(state["rng_counter"]))
        self.shard.buf.load_state_dict(state["shard"])

    def _exchange_stats(self) -> None:
        if self.world > 1:
            self.shard.stats(self._stats)
            dist.all_gather_into_tensor(self._all_flat, self._stats, group=self.group)
        else:
            self.shard.stats(self._all_flat)

    def global_stats(self) -> torch.Tensor:
        """[world, 2] (total priority, live size) of every shard (collective)."""
        self._exchange_stats()
        return self._all_stats.clone()
