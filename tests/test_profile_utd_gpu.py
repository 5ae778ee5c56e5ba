"""The UTD replay-share profiler runs end to end on the engine (B200):
a few environment steps of a synthetic SAC-style learner at UTD 4, with
sane timings and a clean device status."""

import pytest

pytestmark = pytest.mark.gpu


def test_profile_utd_reports_a_replay_share(tmp_path):
    from per_b200 import profile_utd

    r = profile_utd.run(utd=4, batch_size=128, capacity=50_000, steps=5, warmup=2, fill=20_000,
                        trace=str(tmp_path / "trace.json"))
    assert 0.0 < r["replay_share"] < 1.0
    assert r["replay_ms"] > 0 and r["learn_ms"] > 0 and r["step_ms"] > 0
    assert r["status"]["errors"] == 0
    assert (tmp_path / "trace.json").exists()
