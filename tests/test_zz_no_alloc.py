"""The allocation-free update entry point against the regular one (B200).

per_update_priorities_noalloc() exists for callers that cannot allocate
device memory after start-up (a host application that fixes this library's
memory budget, or a latency-critical path where cudaMalloc would stall the
device): it takes its claim and barrier scratch from an array compiled into
the library instead of from the caller's store. It must produce what
per_update_priorities() produces. Both are called here through the C ABI on
two identical stores, twice in a row (the second call finds the scratch as
the first one left it), with batches large enough to take the grid path that
uses the scratch, and once with a small batch.

This file is collected last, and it passes both alone in a fresh process and
after the other tests.
"""

import ctypes

import numpy as np
import pytest
import torch

import cases
from helpers import SUM_RTOL, check_tree, make_buffer
from per_b200 import _lib

pytestmark = pytest.mark.gpu


def _store_without_scratch(buf):
    """The buffer's store descriptor with its claim and barrier scratch removed."""
    s = _lib.Store.from_buffer_copy(buf._store)
    for k in range(_lib.MAX_LEVELS):
        s.claims[k] = None
    s.scratch = None
    s.scratch_bytes = 0
    return s


def _batch(rng, cap, n):
    half = rng.integers(0, cap, n // 2)
    idx = np.concatenate([half, half[rng.integers(0, half.size, n - half.size)]])
    rng.shuffle(idx)
    td = (rng.standard_normal(n) * 3).astype(np.float32)
    return torch.from_numpy(idx.astype(np.int64)).cuda(), torch.from_numpy(td).cuda()


def test_noalloc_update_matches_regular_entry_point():
    rng = np.random.default_rng(41)
    cap = 200_000
    leaves = cases.leaves_abs_normal(rng, cap)
    a = make_buffer(cap, {"x": 1}, None, leaves)
    b = make_buffer(cap, {"x": 1}, None, leaves)
    sb = _store_without_scratch(b)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    for n in (6000, 20000, 300):  # two grid-path calls in a row, then the partitioned path
        idx, td = _batch(rng, cap, n)
        rc_a = _lib.lib.per_update_priorities(a._store_ref, idx.data_ptr(), td.data_ptr(), n, stream)
        rc_b = _lib.lib.per_update_priorities_noalloc(ctypes.byref(sb), idx.data_ptr(),
                                                      td.data_ptr(), n, stream)
        torch.cuda.synchronize()
        assert rc_a == 0 and rc_b == 0, (rc_a, rc_b)
        np.testing.assert_allclose(b.priorities.cpu().numpy(), a.priorities.cpu().numpy(),
                                   rtol=1e-6, atol=0)
        for k in range(1, a.num_levels):
            np.testing.assert_allclose(b.level(k).cpu().numpy(), a.level(k).cpu().numpy(),
                                       rtol=SUM_RTOL, atol=0)
        assert b._max_priority.item() == pytest.approx(a._max_priority.item(), rel=1e-6)
        check_tree(b)
    st = b.status()
    assert st["errors"] == 0 and st["timeouts"] == 0


def test_noalloc_update_at_the_capacity_limit():
    """A store of exactly PER_NOALLOC_MAX_CAPACITY slots fills the array's
    claim regions to their computed bounds: a grid-path batch there gives the
    regular entry point's tree."""
    rng = np.random.default_rng(43)
    cap = _lib.NOALLOC_MAX_CAPACITY
    leaves = cases.leaves_abs_normal(rng, cap)
    a = make_buffer(cap, {"x": 1}, None, leaves)
    b = make_buffer(cap, {"x": 1}, None, leaves)
    sb = _store_without_scratch(b)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    for n in (8192, 5000):
        idx, td = _batch(rng, cap, n)
        idx[:2] = torch.tensor([0, cap - 1])  # the first and the last slot
        rc_a = _lib.lib.per_update_priorities(a._store_ref, idx.data_ptr(), td.data_ptr(), n, stream)
        rc_b = _lib.lib.per_update_priorities_noalloc(ctypes.byref(sb), idx.data_ptr(),
                                                      td.data_ptr(), n, stream)
        torch.cuda.synchronize()
        assert rc_a == 0 and rc_b == 0, (rc_a, rc_b)
        np.testing.assert_allclose(b.priorities.cpu().numpy(), a.priorities.cpu().numpy(),
                                   rtol=1e-6, atol=0)
        for k in range(1, a.num_levels):
            np.testing.assert_allclose(b.level(k).cpu().numpy(), a.level(k).cpu().numpy(),
                                       rtol=SUM_RTOL, atol=0)
    check_tree(b)
    st = b.status()
    assert st["errors"] == 0 and st["timeouts"] == 0


def test_noalloc_rejects_stores_larger_than_its_scratch():
    cap = _lib.NOALLOC_MAX_CAPACITY + 1
    buf = make_buffer(cap, {"x": 1})
    s = _store_without_scratch(buf)
    idx = torch.zeros(4, dtype=torch.int64, device="cuda")
    td = torch.ones(4, device="cuda")
    rc = _lib.lib.per_update_priorities_noalloc(ctypes.byref(s), idx.data_ptr(), td.data_ptr(), 4,
                                                ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 4  # PER_ERR_TOO_LARGE
    assert _lib.lib.per_error_string(rc) == b"size exceeds a supported maximum"
