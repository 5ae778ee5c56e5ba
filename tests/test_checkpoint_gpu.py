"""Checkpoint / resume of the buffer (B200): a buffer restored from a saved
state (through torch.save / torch.load) behaves exactly like the original —
same tree bits, same next draws from sample() (the in-kernel uniform stream
resumes at the saved position), same results after further adds and updates.
The reference keeps no such state (src/triton_per/buffer.py:52-63)."""

import io

import numpy as np
import pytest
import torch

from per_b200 import PERBuffer

pytestmark = pytest.mark.gpu


def _filled(cap, fields, n, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    buf = PERBuffer(cap, fields, device="cuda")
    buf.add({k: torch.randn(n, d, generator=g, device="cuda") for k, d in fields.items()})
    for _ in range(3):
        _, idx, _ = buf.sample(512, 0.4)
        buf.update_priorities(idx, torch.rand(512, generator=g, device="cuda") * 3)
    return buf


@pytest.mark.parametrize("cap,n", [(100_000, 70_000), (50_000, 120_000)])  # partial / wrapped
def test_restored_buffer_continues_identically(cap, n):
    fields = {"obs": 5, "act": 2, "done": 1}
    a = _filled(cap, fields, n, seed=cap)
    blob = io.BytesIO()
    torch.save(a.state_dict(), blob)
    blob.seek(0)
    state = torch.load(blob, weights_only=False)

    b = PERBuffer(cap, fields, device="cuda")
    b.load_state_dict(state)
    assert (b.size, b._cursor) == (a.size, a._cursor)
    for k in range(a.num_levels):
        assert torch.equal(a.level(k), b.level(k)), f"level {k}"
    assert torch.equal(a.storage[: a.size], b.storage[: b.size])
    g = torch.Generator(device="cuda").manual_seed(7)
    for step in range(4):
        va, ia, wa = a.sample(1000, 0.5)
        vb, ib, wb = b.sample(1000, 0.5)
        assert torch.equal(ia, ib) and torch.equal(wa, wb), step
        for k in fields:
            assert torch.equal(va[k], vb[k])
        td = torch.rand(1000, generator=g, device="cuda")
        a.update_priorities(ia, td)
        b.update_priorities(ib, td)
        row = {k: torch.randn(3, d, generator=g, device="cuda") for k, d in fields.items()}
        a.add(row)
        b.add(row)
    assert torch.equal(a.priorities, b.priorities)
    assert a._max_priority.item() == b._max_priority.item()


def test_load_rejects_another_layout():
    a = _filled(10_000, {"x": 3}, 5_000, seed=1)
    with pytest.raises(ValueError):
        PERBuffer(10_000, {"x": 4}, device="cuda").load_state_dict(a.state_dict())
    with pytest.raises(ValueError):
        PERBuffer(20_000, {"x": 3}, device="cuda").load_state_dict(a.state_dict())
