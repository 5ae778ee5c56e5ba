"""GPU-resident prioritized replay buffer on hand-written sm_100a kernels.

Drop-in for triton-per's `PERBuffer` with its `triton` backend
(src/triton_per/buffer.py:23-162): same constructor, attributes, `add`,
`sample(batch_size, beta) -> (views, idx, w)` and
`update_priorities(indices, td_errors)`, and the module constant BLOCK_P.

Storage is one float32[capacity, row_dim] view (rows padded in memory to a
16-byte multiple stride, see per_row_stride, so that rows can be gathered with
bulk copies) and sampling returns zero-copy field views of a freshly allocated
packed [batch, row_dim] output, as in the reference. Priorities live in the reference's two-level store (leaves padded
to BLOCK_P per block plus float32 block sums), widened into a 32-ary sum tree:
the engine also keeps 32-leaf chunk sums (and, above 4M slots, sums of 32
blocks) so that every level of a search is one coalesced warp load.

Every call enqueues CUDA work on the current stream and returns without a host
synchronisation (the reference's add() synchronises through torch.unique; this
one does not). There is no CPU path: a non-CUDA device raises.
"""

from __future__ import annotations

import ctypes
import math

import torch

from . import _lib

try:  # the torch-tensor binding of the hot calls (built beside libper_b200.so)
    from . import _per_torch
except ImportError:  # the ctypes calls below reach the same CUDA library
    _per_torch = None

BLOCK_P = 1024  # priorities per block (reference buffer.py:20)

_BACKENDS = ("triton", "triton-unfused", "b200")
# row element types -> the binding's dtype code
_ROW_DTYPES = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}


def _stream_ptr(device: torch.device):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _current_stream(index: int) -> int:
    """Handle of the current CUDA stream of device `index` (the cheap form of
    torch.cuda.current_stream(index).cuda_stream)."""
    return torch._C._cuda_getCurrentRawStream(index)


class PERBuffer:
    def __init__(
        self,
        capacity: int,
        fields: dict[str, int],  # name -> flattened per-transition dim
        device: str | torch.device = "cuda",
        alpha: float = 0.6,
        eps: float = 1e-6,
        backend: str = "triton",
        storage_dtype: torch.dtype = torch.float32,
    ):
        """`storage_dtype` torch.bfloat16 / torch.float16 keeps the rows in
        16 bits (half the gather bytes; sampled rows come back in that dtype,
        bit for bit; the row width must be even). Not in the reference, whose
        rows are float32 (buffer.py:52)."""
        assert backend in _BACKENDS, (
            f"backend {backend!r}: this engine replaces the reference's triton backends; "
            f"use one of {_BACKENDS}")
        self.capacity = capacity
        self.fields = dict(fields)
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise RuntimeError("per_b200.PERBuffer runs on CUDA devices only (no CPU fallback)")
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        self.alpha = alpha
        self.eps = eps
        self.backend = backend

        self.row_dim = sum(fields.values())
        if storage_dtype not in _ROW_DTYPES:
            raise ValueError(f"storage_dtype must be one of {list(_ROW_DTYPES)}, not {storage_dtype}")
        self.storage_dtype = storage_dtype
        self._elem_bytes = 2 if storage_dtype != torch.float32 else 4
        if self._elem_bytes == 2 and self.row_dim % 2:
            raise ValueError(f"16-bit rows need an even row width, not {self.row_dim}")
        self._offsets: dict[str, tuple[int, int]] = {}
        o = 0
        for name, d in fields.items():
            self._offsets[name] = (o, o + d)
            o += d

        lay = _lib.layout(capacity)
        self._layout = lay
        self.num_blocks = int(lay.num_blocks)
        self.capacity_padded = int(lay.capacity_padded)
        self.log2_blocks = max(1, math.ceil(math.log2(self.num_blocks))) if self.num_blocks > 1 else 0
        self.num_levels = int(lay.num_levels)
        self.top_level = int(lay.top_level)

        dev = self.device
        if self._elem_bytes == 4:
            self.row_stride = int(_lib.lib.per_row_stride(self.row_dim))
        else:  # the recommended stride of the row's 4-byte words, in 16-bit elements
            self.row_stride = 2 * int(_lib.lib.per_row_stride(self.row_dim // 2))
        self._storage = torch.zeros(capacity, self.row_stride, device=dev, dtype=storage_dtype)
        self.storage = self._storage[:, : self.row_dim]
        self._levels = [torch.zeros(int(lay.level_len[k]), device=dev)
                        for k in range(self.num_levels)]
        self.priorities = self._levels[0]
        self.block_sums = self._levels[2][: self.num_blocks]
        self._claims = [torch.zeros(int(lay.level_len[k]), dtype=torch.int32, device=dev)
                        for k in range(self.num_levels)]
        self._size_cursor = torch.zeros(2, dtype=torch.int64, device=dev)
        # device scalar (already ^alpha space) so updates never sync the host
        self._max_priority = torch.ones((), device=dev)
        self._status = torch.zeros(_lib.STATUS_WORDS, dtype=torch.int32, device=dev)
        self._scratch = torch.zeros(int(lay.scratch_bytes), dtype=torch.uint8, device=dev)
        # sample() draws its uniforms inside the kernel (Philox4x32-10, key
        # rng_seed, position in this device word), where the reference calls
        # torch.rand (buffer.py:85); the seed comes from torch's default
        # generator, so torch.manual_seed() makes runs repeatable
        self.rng_seed = int(torch.randint(0, 2**63 - 1, (1,)).item())
        self._rng_counter = torch.zeros(1, dtype=torch.int64, device=dev)
        self._rng_counter_ptr = self._rng_counter.data_ptr()
        self._dev_index = self.device.index
        self._names = tuple(self._offsets)
        self._dims = tuple(b - a for a, b in self._offsets.values())

        self.size = 0
        self._cursor = 0

        s = _lib.Store()
        for k in range(self.num_levels):
            s.levels[k] = self._levels[k].data_ptr()
            s.claims[k] = self._claims[k].data_ptr()
            s.level_len[k] = int(lay.level_len[k])
        s.num_levels = self.num_levels
        s.top_level = self.top_level
        s.capacity = capacity
        s.storage = self._storage.data_ptr()
        s.row_dim = self.row_dim
        s.row_stride = self.row_stride
        s.size_cursor = self._size_cursor.data_ptr()
        s.max_priority = self._max_priority.data_ptr()
        s.status = self._status.data_ptr()
        s.scratch = self._scratch.data_ptr()
        s.scratch_bytes = int(lay.scratch_bytes)
        s.alpha = float(alpha)
        s.eps = float(eps)
        s.elem_bytes = self._elem_bytes
        self._store = s
        self._store_ref = ctypes.byref(s)
        self._engine = (_per_torch.Engine(ctypes.addressof(s), self._dev_index, list(self._names),
                                          list(self._dims), self._rng_counter_ptr,
                                          _ROW_DTYPES[storage_dtype])
                        if _per_torch is not None else None)

    # ------------------------------------------------------------------ add
    def add(self, batch: dict[str, torch.Tensor]) -> None:
        """Insert a batch of transitions (new entries get max priority)."""
        n = next(iter(batch.values())).shape[0]
        if n == 0:
            return
        keep = []
        parts = []
        for name, (a, b) in self._offsets.items():
            t = batch[name].reshape(n, -1)
            if t.shape[1] != b - a:
                raise ValueError(f"field {name!r}: expected {b - a} values per row, got {t.shape[1]}")
            parts.append((t.to(device=self.device, dtype=self.storage_dtype), a, b))
        if self._elem_bytes == 2:  # 16-bit rows move in pairs: one packed field per row
            packed = torch.cat([t for t, _, _ in parts], dim=1).contiguous()
            parts = [(packed, 0, self.row_dim)]
        fields = (_lib.Field * len(parts))()
        for f, (t, a, b) in enumerate(parts):
            if t.stride(1) != 1 or t.stride(0) < t.shape[1]:
                t = t.contiguous()
            keep.append(t)
            fields[f].data = t.data_ptr()
            fields[f].dim = b - a
            fields[f].stride = t.stride(0)
            fields[f].col_offset = a
        with torch.cuda.device(self.device):
            _lib.check("per_add", _lib.lib.per_add(self._store_ref, fields, len(parts), n,
                                                   _stream_ptr(self.device)))
        self._cursor = int((self._cursor + n) % self.capacity)
        self.size = min(self.size + n, self.capacity)

    # --------------------------------------------------------------- sample
    def sample(self, batch_size: int, beta: float = 0.4, out: "SampleOut | None" = None):
        """Returns (fields: dict of views, indices, normalized IS weights).

        With `out` (from sample_out()) the batch is written into that
        caller-owned destination and its views are returned: no allocation
        and no view building per call. The caller orders reuse of `out`
        against readers of its previous contents (same stream, or events)."""
        assert self.size > 0
        if out is not None:
            if out.owner is not self or out.batch != int(batch_size):
                raise ValueError("out was made by sample_out() of another buffer or batch size")
            if self._engine is not None:
                rc = self._engine.sample_into(out.batch, float(beta), self.rng_seed,
                                              out._rows_ptr, out._row_stride, out._idx_ptr,
                                              out._w_ptr)
                if rc:
                    _lib.check("per_sample_fused_rng", rc)
            else:
                self._call("per_sample_fused_rng", _lib.lib.per_sample_fused_rng, self._store_ref,
                           self.rng_seed, self._rng_counter_ptr, out.batch, float(beta),
                           out._rows_ptr, out._row_stride, out._idx_ptr, out._w_ptr)
            return out.fields, out.idx, out.w
        if self._engine is not None:
            rc, views, idx, w = self._engine.sample(int(batch_size), float(beta), self.rng_seed)
            if rc:
                _lib.check("per_sample_fused_rng", rc)
            return views, idx, w
        b = int(batch_size)
        out, idx, w = self._outputs(b)
        self._call("per_sample_fused_rng", _lib.lib.per_sample_fused_rng, self._store_ref,
                   self.rng_seed, self._rng_counter_ptr, b, float(beta), out.data_ptr(),
                   self.row_dim, idx.data_ptr(), w.data_ptr())
        return dict(zip(self._names, out.split(self._dims, dim=1))), idx, w

    def sample_out(self, batch_size: int, rows: torch.Tensor | None = None,
                   idx: torch.Tensor | None = None, w: torch.Tensor | None = None) -> "SampleOut":
        """A reusable destination for sample(batch_size, beta, out=...).

        rows ([batch, row_dim], the storage dtype, unit column stride), idx
        (int64 [batch]) and w (float32 [batch]) may be views into the caller's
        own buffers, e.g. one slot of a [rounds, batch, ...] block that goes to
        the host in one copy; missing ones are allocated here."""
        return SampleOut(self, int(batch_size), rows, idx, w)

    def sample_from_uniforms(self, rand: torch.Tensor, beta: float = 0.4):
        """sample() with caller-provided uniforms in [0, 1) (float32, on the device)."""
        assert self.size > 0
        if rand.dtype != torch.float32 or rand.device != self.device or not rand.is_contiguous():
            rand = rand.to(device=self.device, dtype=torch.float32).contiguous()
        if self._engine is not None:
            rc, views, idx, w = self._engine.sample_from(rand, float(beta))
            if rc:
                _lib.check("per_sample_fused", rc)
            return views, idx, w
        b = rand.numel()
        out, idx, w = self._outputs(b)
        self._call("per_sample_fused", _lib.lib.per_sample_fused, self._store_ref,
                   rand.data_ptr(), b, float(beta), out.data_ptr(), self.row_dim,
                   idx.data_ptr(), w.data_ptr())
        return dict(zip(self._names, out.split(self._dims, dim=1))), idx, w

    def _outputs(self, b: int, extra_idx: int = 0):
        """Fresh [b, row_dim] rows, [b] weights and [b + extra_idx] int64 indices."""
        dev = self.device
        return (torch.empty((b, self.row_dim), device=dev, dtype=self.storage_dtype),
                torch.empty(b + extra_idx, dtype=torch.int64, device=dev),
                torch.empty(b, device=dev))

    def _call(self, name, fn, *args) -> None:
        """fn(*args, stream) on this buffer's device and current stream; raises on error."""
        if torch.cuda.current_device() != self._dev_index:
            with torch.cuda.device(self.device):
                rc = fn(*args, _current_stream(self._dev_index))
        else:
            rc = fn(*args, _current_stream(self._dev_index))
        if rc:
            _lib.check(name, rc)

    # --------------------------------------------------------------- update
    def update_priorities(self, indices: torch.Tensor, td_errors: torch.Tensor) -> None:
        if self._engine is not None:
            # the common case (int64 indices, float32 TD errors, contiguous, on
            # this device) is checked and launched in one C++ call
            rc = self._engine.update_any(indices, td_errors)
            if rc == 0:
                return
            if rc > 0:
                _lib.check("per_update_priorities", rc)
        td = td_errors.detach() if td_errors.requires_grad else td_errors
        if td.dim() != 1:
            td = td.reshape(-1)
        if td.dtype != torch.float32 or td.device != self.device or not td.is_contiguous():
            td = td.to(device=self.device, dtype=torch.float32).contiguous()
        idx = indices if indices.dim() == 1 else indices.reshape(-1)
        if idx.dtype != torch.int64 or idx.device != self.device or not idx.is_contiguous():
            idx = idx.to(device=self.device, dtype=torch.int64).contiguous()
        n = idx.numel()
        if n != td.numel():
            raise ValueError(f"{n} indices but {td.numel()} TD errors")
        if self._engine is not None:
            rc = self._engine.update(idx, td)
            if rc:
                _lib.check("per_update_priorities", rc)
            return
        self._call("per_update_priorities", _lib.lib.per_update_priorities, self._store_ref,
                   idx.data_ptr(), td.data_ptr(), n)

    # ------------------------------------------------------------ utilities
    def rebuild_sums(self) -> None:
        """Recompute every sum level from the leaves (after writing priorities directly)."""
        with torch.cuda.device(self.device):
            _lib.check("per_rebuild_sums", _lib.lib.per_rebuild_sums(
                self._store_ref, _stream_ptr(self.device)))

    def status(self) -> dict[str, int]:
        """Device event counters (synchronises the host)."""
        v = self._status.cpu().tolist()
        return {name: int(v[k]) & 0xFFFFFFFF for k, name in enumerate(_lib.STATUS_NAMES)}

    def clear_status(self) -> None:
        self._status.zero_()

    def recover(self) -> None:
        """Reset the grid-barrier scratch and rebuild the sums after a reported timeout."""
        self._scratch.zero_()
        self.rebuild_sums()

    # ------------------------------------------------------- checkpointing
    STATE_VERSION = 1

    def state_dict(self) -> dict:
        """Everything needed to resume: configuration, rows, leaf priorities,
        size and ring cursor, max priority and the position of the sample()
        uniform stream. (The reference keeps none of this, buffer.py:52-63.)
        The sum levels are not saved: they are exact functions of the leaves
        and load_state_dict() rebuilds them bit for bit. Tensors stay on the
        buffer's device; torch.save() them where they should go."""
        sc = self._size_cursor.tolist()
        return {
            "version": self.STATE_VERSION,
            "capacity": self.capacity,
            "fields": dict(self.fields),
            "storage_dtype": str(self.storage_dtype),
            "alpha": self.alpha,
            "eps": self.eps,
            "size": int(sc[0]),
            "cursor": int(sc[1]),
            "storage": self.storage[: int(sc[0])].clone(),
            "priorities": self.priorities[: self.capacity].clone(),
            "max_priority": self._max_priority.clone(),
            "rng_seed": self.rng_seed,
            "rng_counter": int(self._rng_counter.item()),
        }

    def load_state_dict(self, state: dict) -> None:
        """Restore a state_dict() into a buffer of the same capacity and fields."""
        if state.get("version") != self.STATE_VERSION:
            raise ValueError(f"unsupported buffer state version {state.get('version')!r}")
        if state["capacity"] != self.capacity or dict(state["fields"]) != self.fields:
            raise ValueError("buffer state has a different capacity or field layout")
        if state.get("storage_dtype", "torch.float32") != str(self.storage_dtype):
            raise ValueError("buffer state has a different row dtype")
        if float(state["alpha"]) != float(self.alpha) or float(state["eps"]) != float(self.eps):
            raise ValueError("buffer state has a different alpha or eps")
        n = int(state["size"])
        self._storage.zero_()
        self.storage[:n].copy_(state["storage"].to(self.device))
        self.priorities.zero_()
        self.priorities[: self.capacity].copy_(state["priorities"].to(self.device))
        self._max_priority.copy_(state["max_priority"].to(self.device))
        self._size_cursor.copy_(torch.tensor([n, int(state["cursor"])], dtype=torch.int64))
        self.size = n
        self._cursor = int(state["cursor"])
        self.rng_seed = int(state["rng_seed"])
        self._rng_counter.fill_(int(state["rng_counter"]))
        self._status.zero_()
        self._scratch.zero_()
        self.rebuild_sums()

    def level(self, k: int) -> torch.Tensor:
        """Sums at tree level k (0 = leaves, 1 = 32-leaf chunks, 2 = block sums)."""
        return self._levels[k]


class SampleOut:
    """Caller-owned destination of one sampled batch (device tensors): the
    rows with their per-field views, the indices and the weights. Made by
    PERBuffer.sample_out(); checked once here so that sample(..., out=)
    passes raw pointers only."""

    def __init__(self, owner: PERBuffer, batch: int, rows=None, idx=None, w=None):
        if batch < 1:
            raise ValueError("batch must be positive")
        dev = owner.device
        if rows is None:
            rows = torch.empty((batch, owner.row_dim), device=dev, dtype=owner.storage_dtype)
        if idx is None:
            idx = torch.empty(batch, dtype=torch.int64, device=dev)
        if w is None:
            w = torch.empty(batch, dtype=torch.float32, device=dev)
        if rows.device != dev or idx.device != dev or w.device != dev:
            raise ValueError(f"sample destinations must be on {dev}")
        if rows.dtype != owner.storage_dtype or tuple(rows.shape) != (batch, owner.row_dim) \
                or rows.stride(1) != 1 or rows.stride(0) < owner.row_dim:
            raise ValueError(f"rows must be [{batch}, {owner.row_dim}] {owner.storage_dtype} "
                             "with unit column stride")
        if owner._elem_bytes == 2 and (rows.stride(0) % 2 or rows.data_ptr() % 4):
            raise ValueError("16-bit rows: even row stride and 4-byte aligned start required")
        if idx.dtype != torch.int64 or tuple(idx.shape) != (batch,) or not idx.is_contiguous():
            raise ValueError(f"idx must be a contiguous int64 [{batch}] tensor")
        if w.dtype != torch.float32 or tuple(w.shape) != (batch,) or not w.is_contiguous():
            raise ValueError(f"w must be a contiguous float32 [{batch}] tensor")
        self.owner = owner
        self.batch = batch
        self.rows = rows
        self.idx = idx
        self.w = w
        self.fields = dict(zip(owner._names, rows.split(owner._dims, dim=1)))
        self._rows_ptr = rows.data_ptr()
        self._row_stride = rows.stride(0)
        self._idx_ptr = idx.data_ptr()
        self._w_ptr = w.data_ptr()
