"""TEST INFRASTRUCTURE ONLY - the reference's classic CPU sum tree, restated.

triton-per benchmarks its kernels against a Dopamine-style float64 sum tree
walked on the host (src/triton_per/baselines/cpu_sumtree.py:11-97, selected as
"cpu-sumtree" in bench/bench_sampling.py:23-36 and as the default backend of
bench/profile_utd.py). This module restates it twice:

  SumTreeStore  the same algorithm in C (per_sumtree.c) driven through
                ctypes: one draw and one index at a time, float64 tree.
  PySumTree     the same algorithm as plain Python loops over a numpy tree,
                like the reference's own code, to time what its users see.

Both are pinned to vectors produced by the reference's own SumTree
(tests/golden/sumtree_small.npz, made by tests/golden/make_golden.py). Only
tests/ and the CPU-baseline legs of bench.py and of the UTD profiler use this
module; the engine never does.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
import threading

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "per_sumtree.c")
LIB = os.path.join(HERE, "libper_sumtree.so")

_lib = None
_lock = threading.Lock()
_f64p = np.ctypeslib.ndpointer(np.float64, flags="C_CONTIGUOUS")
_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_i64p = np.ctypeslib.ndpointer(np.int64, flags="C_CONTIGUOUS")


def build(force: bool = False) -> str:
    """Compile per_sumtree.c into libper_sumtree.so (gcc, no fast-math)."""
    if force or not os.path.exists(LIB) or os.path.getmtime(LIB) < os.path.getmtime(SRC):
        cmd = ["gcc", "-O2", "-ffp-contract=off", "-fno-fast-math", "-shared", "-fPIC",
               "-o", LIB + ".tmp", SRC, "-lm"]
        subprocess.run(cmd, check=True)
        os.replace(LIB + ".tmp", LIB)
    return LIB


def lib():
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB):
                build()
            L = ctypes.CDLL(LIB)
            i64, f64 = ctypes.c_int64, ctypes.c_double
            L.sumtree_update.argtypes = [_f64p, i64, i64, f64]
            L.sumtree_find.argtypes = [_f64p, i64, f64]
            L.sumtree_find.restype = i64
            L.sumtree_build.argtypes = [_f64p, i64, _f64p]
            L.sumtree_sample.argtypes = [_f64p, i64, i64, _f64p, i64, f64, _i64p, _f32p, _f64p]
            L.sumtree_update_priorities.argtypes = [_f64p, i64, _i64p, _f32p, i64, f64, f64,
                                                    ctypes.POINTER(ctypes.c_double)]
            L.sumtree_add.argtypes = [_f64p, i64, _f32p, i64, _f32p, i64, f64, _i64p]
            L.sumtree_gather.argtypes = [_f32p, i64, _i64p, i64, _f32p]
            for name in ("sumtree_update", "sumtree_build", "sumtree_sample",
                         "sumtree_update_priorities", "sumtree_add", "sumtree_gather"):
                getattr(L, name).restype = None
            _lib = L
    return _lib


class SumTreeStore:
    """CpuSumTreePER (cpu_sumtree.py:41-97) with its tree walks in C and its
    rows in a host float32 array."""

    def __init__(self, capacity: int, row_dim: int, alpha: float = 0.6, eps: float = 1e-6):
        self.capacity = capacity
        self.row_dim = row_dim
        self.alpha = alpha
        self.eps = eps
        self.tree = np.zeros(2 * capacity, np.float64)
        self.storage = np.zeros((capacity, row_dim), np.float32)
        self.size = 0
        self.cursor = 0
        self.max_priority = 1.0
        self._work = np.empty(0, np.float64)

    def build_from_leaves(self, leaves) -> None:
        """Set-up shortcut: write every leaf at once and sum the inner nodes."""
        lv = np.ascontiguousarray(leaves, np.float64)
        assert lv.size == self.capacity
        lib().sumtree_build(self.tree, self.capacity, lv)

    def total(self) -> float:
        return float(self.tree[1])

    def add(self, rows) -> None:
        r = np.ascontiguousarray(rows, np.float32).reshape(-1, self.row_dim)
        cs = np.array([self.cursor, self.size], np.int64)
        lib().sumtree_add(self.tree, self.capacity, self.storage.reshape(-1), self.row_dim,
                          r.reshape(-1), r.shape[0], self.max_priority, cs)
        self.cursor, self.size = int(cs[0]), int(cs[1])

    def sample_from_uniforms(self, rand, beta: float = 0.4):
        """Returns (idx int64, w float32) for the uniforms rand (float64 in [0, 1))."""
        r = np.ascontiguousarray(rand, np.float64)
        idx = np.empty(r.size, np.int64)
        w = np.empty(r.size, np.float32)
        if self._work.size < r.size:
            self._work = np.empty(r.size, np.float64)
        lib().sumtree_sample(self.tree, self.capacity, self.size, r, r.size, beta, idx, w,
                             self._work)
        return idx, w

    def gather(self, idx, out=None):
        i = np.ascontiguousarray(idx, np.int64)
        if out is None:
            out = np.empty((i.size, self.row_dim), np.float32)
        lib().sumtree_gather(self.storage.reshape(-1), self.row_dim, i, i.size, out.reshape(-1))
        return out

    def update_priorities(self, idx, td) -> None:
        i = np.ascontiguousarray(idx, np.int64).reshape(-1)
        t = np.ascontiguousarray(td, np.float32).reshape(-1)
        mp = ctypes.c_double(self.max_priority)
        lib().sumtree_update_priorities(self.tree, self.capacity, i, t, i.size, self.alpha,
                                        self.eps, ctypes.byref(mp))
        self.max_priority = mp.value


class PySumTree:
    """The reference's SumTree and CpuSumTreePER loops (cpu_sumtree.py:11-35,
    :75-97) as plain Python over a numpy float64 tree, rows on the host."""

    def __init__(self, capacity: int, row_dim: int, alpha: float = 0.6, eps: float = 1e-6):
        self.capacity = capacity
        self.tree = np.zeros(2 * capacity, dtype=np.float64)
        self.storage = np.zeros((capacity, row_dim), np.float32)
        self.alpha = alpha
        self.eps = eps
        self.size = 0
        self.max_priority = 1.0

    def update(self, idx: int, p: float) -> None:
        i = idx + self.capacity
        delta = p - self.tree[i]
        while i >= 1:
            self.tree[i] += delta
            i //= 2

    def find(self, u: float) -> int:
        i = 1
        while i < self.capacity:
            left = 2 * i
            if u <= self.tree[left]:
                i = left
            else:
                u -= self.tree[left]
                i = left + 1
        return i - self.capacity

    def sample_from_uniforms(self, rand, beta: float = 0.4):
        total = float(self.tree[1])
        us = np.asarray(rand, np.float64) * total
        idx = np.empty(us.size, dtype=np.int64)
        probs = np.empty(us.size, dtype=np.float64)
        for j, u in enumerate(us):
            i = min(self.find(u), self.size - 1)
            idx[j] = i
            probs[j] = float(self.tree[i + self.capacity]) / total
        w = (self.size * probs) ** (-beta)
        return idx, (w / w.max()).astype(np.float32), self.storage[idx]

    def update_priorities(self, idx, td) -> None:
        t = np.abs(np.asarray(td, np.float32).reshape(-1))
        for i, v in zip(np.asarray(idx).reshape(-1), t):
            p = (float(v) + self.eps) ** self.alpha
            self.update(int(i), p)
            self.max_priority = max(self.max_priority, p)
