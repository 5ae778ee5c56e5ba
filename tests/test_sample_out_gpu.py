"""sample(..., out=) into caller-owned destinations (B200).

The out= form writes the batch into buffers made once by sample_out() — for
instance one slot of a [rounds, batch, row_dim] block that goes to the host in
one copy — and must return exactly what the allocating sample() returns for
the same position of the in-kernel uniform stream (reference
src/triton_per/buffer.py:82-104 returns fresh tensors per call)."""

import numpy as np
import pytest
import torch

import cases
from helpers import make_buffer

pytestmark = pytest.mark.gpu


def _pair(dtype=torch.float32, cap=200_000, dims=None, seed=5):
    dims = dims or {"obs": 17, "act": 6, "rew": 1, "next_obs": 17, "done": 1}
    out = []
    for _ in range(2):  # two identical buffers: one samples with out=, one without
        rng = np.random.default_rng(seed)
        rows = {k: rng.standard_normal((cap, d), dtype=np.float32) for k, d in dims.items()}
        buf = make_buffer(cap, dims, rows, cases.leaves_abs_normal(rng, cap), storage_dtype=dtype)
        buf.rng_seed = 0xDEC0DE
        buf._rng_counter.fill_(0)
        out.append(buf)
    return out


@pytest.mark.parametrize("batch", [1, 256, 4099])
def test_out_equals_allocating_sample(batch):
    a, b = _pair()
    so = b.sample_out(batch)
    for _ in range(3):
        fa, ia, wa = a.sample(batch, 0.6)
        fb, ib, wb = b.sample(batch, 0.6, out=so)
        assert ib is so.idx and wb is so.w
        assert torch.equal(ia, ib)
        assert torch.equal(wa, wb)
        for k in fa:
            assert torch.equal(fa[k], fb[k])
        td = torch.rand(batch, device="cuda") + 0.1
        a.update_priorities(ia, td)
        b.update_priorities(ib, td)


def test_slots_of_one_block():
    a, b = _pair()
    rounds, batch = 4, 256
    rows = torch.full((rounds, batch, a.row_dim + 3), -7.0, device="cuda")[:, :, :a.row_dim]
    idx = torch.empty(rounds, batch, dtype=torch.int64, device="cuda")
    w = torch.empty(rounds, batch, device="cuda")
    outs = [b.sample_out(batch, rows=rows[r], idx=idx[r], w=w[r]) for r in range(rounds)]
    ref = []
    for r in range(rounds):
        fa, ia, wa = a.sample(batch, 0.4)
        ref.append((torch.cat(list(fa.values()), 1), ia, wa))
        b.sample(batch, 0.4, out=outs[r])
    for r in range(rounds):
        assert torch.equal(rows[r], ref[r][0])
        assert torch.equal(idx[r], ref[r][1])
        assert torch.equal(w[r], ref[r][2])


def test_bf16_rows_out():
    a, b = _pair(dtype=torch.bfloat16, dims={"obs": 10, "act": 4})
    so = b.sample_out(300)
    fa, ia, wa = a.sample(300, 0.4)
    fb, ib, wb = b.sample(300, 0.4, out=so)
    assert torch.equal(ia, ib) and torch.equal(wa, wb)
    assert torch.equal(fa["obs"], fb["obs"]) and torch.equal(fa["act"], fb["act"])


def test_out_of_another_shape_is_rejected():
    a, b = _pair(cap=50_000)
    so = a.sample_out(64)
    with pytest.raises(ValueError):
        a.sample(65, 0.4, out=so)
    with pytest.raises(ValueError):
        b.sample(64, 0.4, out=so)
    with pytest.raises(ValueError):
        a.sample_out(64, rows=torch.empty(64, a.row_dim, device="cuda")[:, :-1])
    with pytest.raises(ValueError):
        a.sample_out(64, idx=torch.empty(64, dtype=torch.int32, device="cuda"))


def test_out_through_the_ctypes_path():
    """The out= form without the torch binding (C ABI through ctypes)."""
    a, b = _pair(cap=80_000)
    b._engine = None
    so = b.sample_out(512)
    fa, ia, wa = a.sample(512, 0.4)
    fb, ib, wb = b.sample(512, 0.4, out=so)
    assert torch.equal(ia, ib) and torch.equal(wa, wb)
    for k in fa:
        assert torch.equal(fa[k], fb[k])
