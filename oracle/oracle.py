"""TEST INFRASTRUCTURE ONLY - the oracle of the replay engine.

CPU restatement of triton-per's `torch` backend (src/triton_per/buffer.py:66-79
add, :82-105 sample, :133-145 update_priorities) in C (per_oracle.c), driven
through ctypes with numpy arrays. Only tests/, __graft_entry__.smoke() and the
CPU-baseline legs of bench.py may import this module; the engine never does.

Pinned against vectors produced by the reference itself (tests/golden/,
made by tests/golden/make_golden.py, which imports the reference package).
"""

from __future__ import annotations

import ctypes
import os
import subprocess
import threading

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "per_oracle.c")
LIB = os.path.join(HERE, "libper_oracle.so")
BLOCK_P = 1024

_lib = None
_lock = threading.Lock()

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_i64p = np.ctypeslib.ndpointer(np.int64, flags="C_CONTIGUOUS")


def build(force: bool = False) -> str:
    """Compile per_oracle.c into libper_oracle.so (gcc, OpenMP, no fast-math)."""
    if force or not os.path.exists(LIB) or os.path.getmtime(LIB) < os.path.getmtime(SRC):
        cmd = ["gcc", "-O2", "-fopenmp", "-ffp-contract=off", "-fno-fast-math",
               "-shared", "-fPIC", "-o", LIB, SRC, "-lm"]
        subprocess.run(cmd, check=True)
    return LIB


def lib():
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB):
                build()
            L = ctypes.CDLL(LIB)
            i64, i32, f32 = ctypes.c_int64, ctypes.c_int, ctypes.c_float
            L.oracle_cumsum.argtypes = [_f32p, i64, _f32p, i32]
            L.oracle_sample_from_csum.argtypes = [_f32p, _f32p, i64, i64, _f32p, i64, f32,
                                                  _i64p, _f32p, ctypes.c_void_p, i32]
            L.oracle_sample.argtypes = [_f32p, i64, i64, _f32p, i64, f32, _i64p, _f32p,
                                        ctypes.c_void_p, i32]
            L.oracle_weights_for.argtypes = [_f32p, f32, i64, _i64p, i64, f32, _f32p]
            L.oracle_block_sums.argtypes = [_f32p, i64, _f32p]
            L.oracle_update.argtypes = [_f32p, _f32p, i64, _i64p, _f32p, i64, f32, f32,
                                        ctypes.POINTER(ctypes.c_float)]
            L.oracle_add.argtypes = [_f32p, i64, _f32p, _f32p, i64, i64, _f32p, i64, f32, _i64p]
            for name in ("oracle_cumsum", "oracle_sample_from_csum", "oracle_sample",
                         "oracle_weights_for", "oracle_block_sums", "oracle_update",
                         "oracle_add"):
                getattr(L, name).restype = None
            _lib = L
    return _lib


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def _i64(a):
    return np.ascontiguousarray(a, dtype=np.int64)


def cumsum(p, nthreads: int = 1) -> np.ndarray:
    """torch.cumsum(p) on CPU (buffer.py:98): double accumulation, float32 out."""
    p = _f32(p)
    out = np.empty_like(p)
    lib().oracle_cumsum(p, p.size, out, nthreads)
    return out


def sample(priorities, capacity: int, size: int, rand, beta: float, nthreads: int = 1):
    """buffer.py:96-105 + :92. Returns (idx int64, w float32 normalised, csum)."""
    p = _f32(priorities)
    r = _f32(rand)
    csum = np.empty(capacity, np.float32)
    idx = np.empty(r.size, np.int64)
    w = np.empty(r.size, np.float32)
    lib().oracle_sample(p, capacity, size, r, r.size, beta, idx, w,
                        csum.ctypes.data_as(ctypes.c_void_p), nthreads)
    return idx, w, csum


def sample_from_csum(priorities, csum, capacity: int, size: int, rand, beta: float,
                     nthreads: int = 1):
    """Sample with a precomputed cumsum; returns (idx, w, w_unnormalised)."""
    p, c, r = _f32(priorities), _f32(csum), _f32(rand)
    idx = np.empty(r.size, np.int64)
    w = np.empty(r.size, np.float32)
    wu = np.empty(r.size, np.float32)
    lib().oracle_sample_from_csum(p, c, capacity, size, r, r.size, beta, idx, w,
                                  wu.ctypes.data_as(ctypes.c_void_p), nthreads)
    return idx, w, wu


def weights_for(priorities, total: float, size: int, idx, beta: float) -> np.ndarray:
    """IS weights (buffer.py:102-103, :92) of the given indices."""
    p, i = _f32(priorities), _i64(idx)
    w = np.empty(i.size, np.float32)
    lib().oracle_weights_for(p, np.float32(total), size, i, i.size, beta, w)
    return w


def block_sums(priorities) -> np.ndarray:
    p = _f32(priorities)
    nb = p.size // BLOCK_P
    out = np.empty(nb, np.float32)
    lib().oracle_block_sums(p, nb, out)
    return out


def tree_sums(priorities, capacity: int, level: int) -> np.ndarray:
    """Exact float64 sums of 32**level consecutive leaves (live nodes only)."""
    p = np.asarray(priorities, np.float64)[:capacity]
    span = 32 ** level
    n = -(-capacity // span)
    pad = np.zeros(n * span, np.float64)
    pad[:capacity] = p
    return pad.reshape(n, span).sum(axis=1)


class OracleStore:
    """numpy mirror of a PERBuffer on the torch backend (buffer.py:24-63)."""

    def __init__(self, capacity: int, fields: dict[str, int], alpha: float = 0.6,
                 eps: float = 1e-6):
        self.capacity = capacity
        self.fields = dict(fields)
        self.alpha = alpha
        self.eps = eps
        self.row_dim = sum(fields.values())
        self._offsets = {}
        o = 0
        for name, d in fields.items():
            self._offsets[name] = (o, o + d)
            o += d
        self.num_blocks = -(-capacity // BLOCK_P)
        self.capacity_padded = self.num_blocks * BLOCK_P
        self.storage = np.zeros((capacity, self.row_dim), np.float32)
        self.priorities = np.zeros(self.capacity_padded, np.float32)
        self.block_sums = np.zeros(self.num_blocks, np.float32)
        self.max_priority = np.float32(1.0)
        self.size = 0
        self.cursor = 0

    def add(self, batch: dict) -> None:
        n = next(iter(batch.values())).shape[0]
        rows = np.zeros((n, self.row_dim), np.float32)
        for name, (a, b) in self._offsets.items():
            rows[:, a:b] = np.asarray(batch[name], np.float32).reshape(n, -1)
        cs = np.array([self.cursor, self.size], np.int64)
        lib().oracle_add(self.storage.reshape(-1), self.row_dim, self.priorities,
                         self.block_sums, self.capacity, self.num_blocks,
                         np.ascontiguousarray(rows.reshape(-1)), n,
                         np.float32(self.max_priority), cs)
        self.cursor, self.size = int(cs[0]), int(cs[1])

    def set_priorities(self, leaves) -> None:
        """Write leaves directly, then recompute every block sum exactly."""
        self.priorities[:] = _f32(leaves)
        self.block_sums[:] = block_sums(self.priorities)

    def sample_from_uniforms(self, rand, beta: float = 0.4):
        idx, w, csum = sample(self.priorities, self.capacity, self.size, rand, beta)
        return idx, w, csum

    def update_priorities(self, idx, td) -> None:
        mp = ctypes.c_float(float(self.max_priority))
        lib().oracle_update(self.priorities, self.block_sums, self.num_blocks, _i64(idx),
                            _f32(np.asarray(td).reshape(-1)), int(np.asarray(idx).size),
                            self.alpha, self.eps, ctypes.byref(mp))
        self.max_priority = np.float32(mp.value)


def ulp32(x) -> np.ndarray:
    x = np.abs(np.asarray(x, np.float32))
    return np.spacing(x).astype(np.float64)


def classify_indices(idx_test, idx_oracle, rand, csum, size: int):
    """Compare sampled indices with the oracle's.

    A mismatch is EXCUSED when u = rand * total lies within 1 ulp of the
    oracle's prefix boundary between the two indices (csum at the smaller
    index): the two searches then straddle a float32 tie of the prefix sum.
    Returns (n_equal, n_excused, bad_positions).
    """
    it = np.asarray(idx_test, np.int64)
    io = np.asarray(idx_oracle, np.int64)
    csum = np.asarray(csum, np.float32)
    total = csum[-1]
    u = (np.asarray(rand, np.float32) * total).astype(np.float32)
    diff = np.nonzero(it != io)[0]
    excused = np.zeros(diff.size, bool)
    if diff.size:
        lo = np.minimum(it[diff], io[diff])
        lo = np.clip(lo, 0, csum.size - 1)
        b = csum[lo].astype(np.float64)
        excused = np.abs(u[diff].astype(np.float64) - b) <= ulp32(b)
    return int(it.size - diff.size), int(excused.sum()), diff[~excused]


# ------------------------------------------------------------------ Philox
PHILOX_M0, PHILOX_M1 = 0xD2511F53, 0xCD9E8D57
PHILOX_W0, PHILOX_W1 = 0x9E3779B9, 0xBB67AE85


def philox4x32_10(ctr: np.ndarray, key: tuple[int, int]) -> np.ndarray:
    """Philox4x32-10 (Salmon, Moraes, Dror, Shaw, "Parallel random numbers: as
    easy as 1, 2, 3", SC 2011) on uint32 counters ctr[..., 4]; returns the
    uint32 outputs [..., 4]. Vectorised numpy restatement of the published
    round function: two 32x32->64 products per round, keys bumped by the Weyl
    constants. The engine's sample() uses it in place of the reference's
    torch.rand (src/triton_per/buffer.py:85)."""
    c = ctr.astype(np.uint64) & 0xFFFFFFFF
    c0, c1, c2, c3 = c[..., 0], c[..., 1], c[..., 2], c[..., 3]
    k0, k1 = np.uint64(key[0] & 0xFFFFFFFF), np.uint64(key[1] & 0xFFFFFFFF)
    mask = np.uint64(0xFFFFFFFF)
    for _ in range(10):
        p0 = np.uint64(PHILOX_M0) * c0
        p1 = np.uint64(PHILOX_M1) * c2
        c0, c1, c2, c3 = ((p1 >> np.uint64(32)) ^ c1 ^ k0, p1 & mask,
                          (p0 >> np.uint64(32)) ^ c3 ^ k1, p0 & mask)
        k0 = (k0 + np.uint64(PHILOX_W0)) & mask
        k1 = (k1 + np.uint64(PHILOX_W1)) & mask
    return np.stack([c0, c1, c2, c3], axis=-1).astype(np.uint32)


def philox_uniforms(seed: int, start: int, n: int) -> np.ndarray:
    """Uniform j of the engine's stream `seed`: counter (lo(j), hi(j), 0, 0),
    key (lo(seed), hi(seed)), top 24 bits of output word 0 times 2^-24."""
    j = np.arange(start, start + n, dtype=np.uint64)
    ctr = np.zeros((n, 4), np.uint64)
    ctr[:, 0] = j & np.uint64(0xFFFFFFFF)
    ctr[:, 1] = j >> np.uint64(32)
    out = philox4x32_10(ctr, (seed & 0xFFFFFFFF, (seed >> 32) & 0xFFFFFFFF))
    return ((out[:, 0] >> 8).astype(np.float32) * np.float32(2.0 ** -24)).astype(np.float32)
