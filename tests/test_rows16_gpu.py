"""16-bit row storage (B200): `PERBuffer(..., storage_dtype=torch.bfloat16 /
torch.float16)` keeps the rows in 16 bits (half the gather bytes; not in the
reference, whose rows are float32, src/triton_per/buffer.py:52). Sampling is
unchanged — the same indices and IS weights as a float32 buffer with the
same priorities and uniforms — and the gathered rows are the stored 16-bit
rows bit for bit, through both gather paths (staged rows and wide rows)."""

import numpy as np
import pytest
import torch

import cases
from per_b200 import PERBuffer

pytestmark = pytest.mark.gpu


def _pair(cap, fields, dtype, seed):
    rng = np.random.default_rng(seed)
    rows = {k: torch.from_numpy(rng.standard_normal((cap, d), dtype=np.float32)).cuda()
            for k, d in fields.items()}
    leaves = torch.from_numpy(cases.leaves_abs_normal(rng, cap)).cuda()
    bufs = []
    for dt in (torch.float32, dtype):
        b = PERBuffer(cap, fields, device="cuda", storage_dtype=dt)
        b.add(rows)
        b.priorities[:cap] = leaves
        b.rebuild_sums()
        bufs.append(b)
    return bufs, rows


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("fields", [{"obs": 32, "action": 8, "reward": 1, "next_obs": 32, "done": 1},
                                    {"img": 6000}])  # 74 (staged rows), 6000 (wide-row kernel)
def test_16bit_rows_sample_like_float32(dtype, fields):
    cap = 20_000 if "img" in fields else 200_000
    (b32, b16), rows = _pair(cap, fields, dtype, seed=len(fields))
    packed16 = torch.cat([rows[k] for k in fields], dim=1).to(dtype)
    assert b16.storage.dtype == dtype and torch.equal(b16.storage[:cap], packed16)
    for batch in (256, 5000):
        rand = torch.rand(batch, device="cuda")
        v32, i32, w32 = b32.sample_from_uniforms(rand, 0.4)
        v16, i16, w16 = b16.sample_from_uniforms(rand, 0.4)
        assert torch.equal(i16, i32) and torch.equal(w16, w32)
        for k in fields:
            assert v16[k].dtype == dtype
            assert torch.equal(v16[k], rows[k][i16].to(dtype))
    _, idx, _ = b16.sample(1000)
    b16.update_priorities(idx, torch.rand(1000, device="cuda"))
    assert b16.status()["errors"] == 0


def test_16bit_rows_need_an_even_width():
    with pytest.raises(ValueError):
        PERBuffer(1000, {"a": 3, "b": 2}, device="cuda", storage_dtype=torch.bfloat16)


def test_16bit_checkpoint_round_trip():
    (_, b16), _ = _pair(10_000, {"x": 6}, torch.bfloat16, seed=3)
    c = PERBuffer(10_000, {"x": 6}, device="cuda", storage_dtype=torch.bfloat16)
    c.load_state_dict(b16.state_dict())
    v1, i1, w1 = b16.sample(512)
    v2, i2, w2 = c.sample(512)
    assert torch.equal(i1, i2) and torch.equal(v1["x"], v2["x"])
    with pytest.raises(ValueError):
        PERBuffer(10_000, {"x": 6}, device="cuda").load_state_dict(b16.state_dict())
