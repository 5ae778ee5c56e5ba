"""In-kernel uniforms of sample() (B200).

PERBuffer.sample() draws its uniforms inside the fused kernel from a
Philox4x32-10 stream instead of launching torch.rand as the reference does
(src/triton_per/buffer.py:85). The stream must be exactly the oracle's
restatement of the published generator: a sample through
per_sample_fused_rng equals per_sample_fused on the oracle's uniforms bit for
bit, the device counter advances by the batch, and CUDA-graph replays
continue the stream."""

import ctypes

import numpy as np
import pytest
import torch

import cases
from helpers import make_buffer
from oracle import oracle
from per_b200 import _lib

pytestmark = pytest.mark.gpu


def _fused(buf, rand):
    b = rand.numel()
    out = torch.empty(b, buf.row_dim, device="cuda")
    idx = torch.empty(b, dtype=torch.int64, device="cuda")
    w = torch.empty(b, device="cuda")
    rc = _lib.lib.per_sample_fused(buf._store_ref, rand.data_ptr(), b, 0.4, out.data_ptr(),
                                   buf.row_dim, idx.data_ptr(), w.data_ptr(),
                                   ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0
    return out, idx, w


@pytest.mark.parametrize("batch", [1, 256, 5000, 65536])
def test_in_kernel_uniforms_equal_the_oracle_stream(batch):
    rng = np.random.default_rng(batch)
    cap = 300_000
    rows = {"x": rng.standard_normal((cap, 9), dtype=np.float32)}
    buf = make_buffer(cap, {"x": 9}, rows, cases.leaves_abs_normal(rng, cap))
    buf.rng_seed = 0x1234_5678_9ABC_DEF1
    start = 2**32 - 100  # the draw counter crosses the 32-bit boundary
    buf._rng_counter.fill_(start)
    for call in range(2):
        views, idx, w = buf.sample(batch, 0.4)
        u = oracle.philox_uniforms(buf.rng_seed, start + call * batch, batch)
        out2, idx2, w2 = _fused(buf, torch.from_numpy(u).cuda())
        assert torch.equal(idx, idx2)
        assert torch.equal(w, w2)
        assert torch.equal(views["x"], out2)
        assert int(buf._rng_counter.item()) == start + (call + 1) * batch


def test_graph_replays_continue_the_stream():
    rng = np.random.default_rng(3)
    cap = 100_000
    buf = make_buffer(cap, {"x": 4}, {"x": rng.standard_normal((cap, 4), dtype=np.float32)},
                      cases.leaves_abs_normal(rng, cap))
    batch = 512
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        buf.sample(batch, 0.4)  # warm-up (loads the module, sets attributes)
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    start = int(buf._rng_counter.item())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        _, idx_g, _ = buf.sample(batch, 0.4)
    seen = []
    for _ in range(3):
        g.replay()
        seen.append(idx_g.clone())
    torch.cuda.synchronize()
    assert int(buf._rng_counter.item()) == start + 3 * batch
    for k, idx in enumerate(seen):
        u = oracle.philox_uniforms(buf.rng_seed, start + k * batch, batch)
        _, idx2, _ = _fused(buf, torch.from_numpy(u).cuda())
        assert torch.equal(idx, idx2)
