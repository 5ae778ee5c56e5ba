"""Distributional correctness on the B200 engine: empirical sampling
frequencies against P(i) = p_i / sum(p) (chi-square), and IS weights against
the analytic (N P(i))^-beta / max. Same test bodies and bars as the
reference's tests/test_distribution.py (:44-113)."""

import pytest
import torch
from scipy import stats

from per_b200 import PERBuffer

pytestmark = pytest.mark.gpu


def fill_with_known_priorities(buf, n, seed=0):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(n, 4, generator=g).to(buf.device)
    buf.add({"x": x})
    td = torch.rand(n, generator=g).to(buf.device) * 10 + 0.01
    buf.update_priorities(torch.arange(n, device=buf.device), td)
    expected_p = (td.cpu().double().abs() + buf.eps) ** buf.alpha
    return expected_p / expected_p.sum()


def test_sampling_matches_distribution():
    n = 512
    buf = PERBuffer(4096, {"x": 4}, device="cuda")
    probs = fill_with_known_priorities(buf, n)
    draws, bs = 400_000, 4096
    counts = torch.zeros(n, dtype=torch.long)
    for _ in range(draws // bs):
        _, idx, _ = buf.sample(bs)
        counts += torch.bincount(idx.cpu(), minlength=n)
    expected = (probs * counts.sum().item()).numpy()
    assert expected.min() > 5
    chi2, p_value = stats.chisquare(counts.numpy(), expected)
    print(f"CHISQ b200: chi2={chi2:.1f} p={p_value:.4f}")
    assert p_value > 0.001


def test_is_weights():
    n = 256
    buf = PERBuffer(1024, {"x": 4}, device="cuda")
    probs = fill_with_known_priorities(buf, n)
    beta = 0.5
    _, idx, w = buf.sample(2048, beta=beta)
    ref = (n * probs[idx.cpu()]) ** (-beta)
    ref = ref / ref.max()
    torch.testing.assert_close(w.cpu().double(), ref, rtol=1e-3, atol=1e-4)


def test_sampling_binned_large_buffer():
    """1e6 slots, 1e4-slot bins, after 1500 update rounds (reference :80-113)."""
    n = 1_000_000
    buf = PERBuffer(n, {"x": 1}, device="cuda")
    chunk = 200_000
    for _ in range(0, n, chunk):
        buf.add({"x": torch.zeros(chunk, 1, device="cuda")})
    g = torch.Generator(device="cuda").manual_seed(1)
    for _ in range(1500):
        idx = torch.randint(0, n, (1024,), device="cuda", generator=g)
        buf.update_priorities(idx, torch.rand(1024, device="cuda", generator=g) * 5)
    probs = (buf.priorities[:n].double() / buf.priorities[:n].double().sum()).cpu()
    bin_size = 10_000
    bin_mass = probs.reshape(-1, bin_size).sum(dim=1).numpy()
    counts = torch.zeros(n // bin_size, dtype=torch.long)
    for _ in range(1_000_000 // 4096):
        _, idx, _ = buf.sample(4096)
        counts += torch.bincount((idx // bin_size).cpu(), minlength=n // bin_size)
    expected = bin_mass * counts.sum().item()
    assert expected.min() > 5
    chi2, p_value = stats.chisquare(counts.numpy(), expected)
    print(f"CHISQ-LARGE b200: chi2={chi2:.1f} p={p_value:.4f}")
    assert p_value > 0.001
    # sums stay exact without any periodic refresh
    exact = buf.priorities.view(buf.num_blocks, 1024).double().sum(dim=1)
    rel = ((buf.block_sums.double() - exact).abs() / exact.clamp(min=1e-12)).max().item()
    assert rel < 1e-6


def test_sampling_64m_single_store():
    """64M slots (four-level tree, top level above the blocks): block-level chi-square."""
    n = 64_000_000
    buf = PERBuffer(n, {"x": 1}, device="cuda")
    assert buf.num_levels == 4 and buf.top_level == 3
    g = torch.Generator(device="cuda").manual_seed(5)
    buf.add({"x": torch.zeros(n, 1, device="cuda")})
    leaves = torch.empty(n, device="cuda").log_normal_(0.0, 1.0, generator=g)
    buf.priorities[:n] = leaves
    buf.rebuild_sums()
    bin_size = 1_000_000
    mass = (buf.priorities[:n].double().reshape(-1, bin_size).sum(1) /
            buf.priorities[:n].double().sum()).cpu().numpy()
    counts = torch.zeros(n // bin_size, dtype=torch.long, device="cuda")
    for _ in range(100):
        _, idx, _ = buf.sample(65536)
        counts += torch.bincount(idx // bin_size, minlength=n // bin_size)
    counts = counts.cpu()
    expected = mass * counts.sum().item()
    chi2, p_value = stats.chisquare(counts.numpy(), expected)
    print(f"CHISQ-64M b200: chi2={chi2:.1f} p={p_value:.4f}")
    assert p_value > 0.001
