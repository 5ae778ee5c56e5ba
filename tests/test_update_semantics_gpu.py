"""Priority-update semantics on the B200 engine (reference
tests/test_update_semantics.py:19-58): block sums stay consistent, duplicates
resolve to one submitted value (the last one), circular overwrite keeps sums
correct, sampled rows equal stored rows."""

import pytest
import torch

from per_b200 import BLOCK_P, PERBuffer

pytestmark = pytest.mark.gpu
DEV = "cuda"


def consistent(buf):
    ref = buf.priorities.view(buf.num_blocks, BLOCK_P).sum(dim=1)
    torch.testing.assert_close(buf.block_sums, ref, rtol=1e-5, atol=1e-5)


def test_block_sums_after_updates():
    buf = PERBuffer(BLOCK_P * 3, {"x": 2}, device=DEV)
    buf.add({"x": torch.randn(2000, 2).to(DEV)})
    consistent(buf)
    idx = torch.randint(0, 2000, (512,), device=DEV)
    buf.update_priorities(idx, torch.rand(512, device=DEV) * 5)
    consistent(buf)


def test_duplicate_indices():
    buf = PERBuffer(BLOCK_P, {"x": 2}, device=DEV)
    buf.add({"x": torch.randn(100, 2).to(DEV)})
    idx = torch.zeros(64, dtype=torch.int64, device=DEV)
    buf.update_priorities(idx, torch.linspace(0.1, 5, 64, device=DEV))
    consistent(buf)
    p0 = buf.priorities[0].item()
    candidates = (torch.linspace(0.1, 5, 64).abs() + buf.eps) ** buf.alpha
    assert (candidates - p0).abs().min() < 1e-5
    assert abs(candidates[-1].item() - p0) < 1e-6  # last occurrence wins


def test_circular_overwrite():
    buf = PERBuffer(256, {"x": 1}, device=DEV)
    for _ in range(5):
        buf.add({"x": torch.randn(100, 1).to(DEV)})
    assert buf.size == 256
    consistent(buf)


def test_sample_returns_stored_rows():
    buf = PERBuffer(512, {"a": 3, "b": 1}, device=DEV)
    a = torch.randn(200, 3).to(DEV)
    b = torch.arange(200, dtype=torch.float32).reshape(-1, 1).to(DEV)
    buf.add({"a": a, "b": b})
    views, idx, _ = buf.sample(64)
    torch.testing.assert_close(views["a"], a[idx])
    torch.testing.assert_close(views["b"], b[idx])


def test_max_priority_tracking_and_new_entries():
    buf = PERBuffer(4096, {"x": 1}, device=DEV)
    buf.add({"x": torch.zeros(10, 1, device=DEV)})
    assert torch.all(buf.priorities[:10] == 1.0)
    buf.update_priorities(torch.tensor([3], device=DEV), torch.tensor([-100.0], device=DEV))
    mp = (100.0 + 1e-6) ** 0.6
    assert buf._max_priority.item() == pytest.approx(mp, rel=1e-6)
    buf.add({"x": torch.zeros(5, 1, device=DEV)})
    torch.testing.assert_close(buf.priorities[10:15], torch.full((5,), mp, device=DEV),
                               rtol=1e-6, atol=0)
    consistent(buf)


def test_graph_capture_of_a_utd_round():
    """sample -> update -> add captured into one CUDA graph and replayed."""
    buf = PERBuffer(100_000, {"x": 3}, device=DEV)
    buf.add({"x": torch.randn(100_000, 3, device=DEV)})
    td = torch.rand(256, device=DEV)
    row = torch.randn(1, 3, device=DEV)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(3):
            _, idx, _ = buf.sample(256)
            buf.update_priorities(idx, td)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        _, idx, w = buf.sample(256)
        buf.update_priorities(idx, td)
        buf.add({"x": row})
    for _ in range(50):
        g.replay()
    torch.cuda.synchronize()
    consistent(buf)
    st = buf.status()
    assert st["errors"] == 0 and st["timeouts"] == 0
    assert buf._size_cursor.tolist()[0] == 100_000
