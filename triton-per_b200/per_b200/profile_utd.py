"""Replay share of a high-UTD training step on the B200 engine.

    python -m per_b200.profile_utd --utd 32 --batch-size 256 --steps 60 [--num-q 10] [--trace out.json]

The caller context of the hot path (the reference measures it with
bench/profile_utd.py:76-97): a SAC-style update phase — an MLP actor and
`num_q` MLP critics (two hidden layers of 256), Adam — where every gradient
step samples a prioritized batch, computes TD errors and writes them back as
priorities, `utd` times per environment step, with one new transition added
per environment step. It reports the fraction of step time spent in the
replay calls (sample + update_priorities).

Unlike a host timer around synchronised calls, each phase is bracketed by
CUDA events on the stream and nothing synchronises inside the loop, so the
share is the replay's part of the device timeline as the learner actually
runs it (the host enqueues ahead). `--trace` exports a torch.profiler Chrome
trace of a few steps.

run(buffer=..., timing="wall") drives any buffer with the PERBuffer API (for
instance a host-side baseline whose priorities live on the CPU) and times
each phase with the host clock around synchronised calls, the method of the
reference's profiler (bench/profile_utd.py:76-97), so that engines whose work
is partly on the host compare on equal terms.
"""

from __future__ import annotations

import argparse
import json
import time

import torch
import torch.nn as nn

from .buffer import PERBuffer


def mlp(i: int, o: int, h: int = 256) -> nn.Module:
    return nn.Sequential(nn.Linear(i, h), nn.ReLU(), nn.Linear(h, h), nn.ReLU(), nn.Linear(h, o))


class Learner:
    """Actor + critics with one optimiser; step() returns |TD| per sample."""

    def __init__(self, obs_dim: int, act_dim: int, num_q: int, device):
        self.actor = mlp(obs_dim, act_dim).to(device)
        self.qs = nn.ModuleList([mlp(obs_dim + act_dim, 1) for _ in range(num_q)]).to(device)
        self.opt = torch.optim.Adam(list(self.actor.parameters()) + list(self.qs.parameters()),
                                    lr=3e-4)

    def step(self, batch: dict, w: torch.Tensor) -> torch.Tensor:
        obs, act, rew = batch["obs"], batch["action"], batch["reward"].squeeze(-1)
        qin = torch.cat([obs, act], dim=-1)
        tds = [q(qin).squeeze(-1) - rew for q in self.qs]
        loss = sum((w * td.pow(2)).mean() for td in tds) + 1e-3 * self.actor(obs).pow(2).mean()
        self.opt.zero_grad(set_to_none=True)
        loss.backward()
        self.opt.step()
        return tds[0].detach().abs()


def run(utd: int = 32, batch_size: int = 256, capacity: int = 1_000_000, obs_dim: int = 32,
        act_dim: int = 8, num_q: int = 2, steps: int = 60, warmup: int = 10, fill: int = 200_000,
        device: str = "cuda", trace: str | None = None, seed: int = 0, buffer=None,
        timing: str = "events") -> dict:
    """buffer: a buffer with the PERBuffer API built for these fields and
    capacity (default: this engine's PERBuffer). timing "events": CUDA events
    on the stream, nothing synchronised; "wall": host clock around
    synchronised phases."""
    if timing not in ("events", "wall"):
        raise ValueError(f"timing must be 'events' or 'wall', not {timing!r}")
    torch.manual_seed(seed)
    dev = torch.device(device)
    fields = {"obs": obs_dim, "action": act_dim, "reward": 1, "next_obs": obs_dim, "done": 1}
    buf = buffer if buffer is not None else PERBuffer(capacity, fields, device=dev)
    n = min(capacity, fill)
    buf.add({k: torch.randn(n, d, device=dev) for k, d in fields.items()})
    learner = Learner(obs_dim, act_dim, num_q, dev)
    new_row = {k: torch.randn(1, d, device=dev) for k, d in fields.items()}

    stream = torch.cuda.current_stream(dev)
    marks = []  # per gradient step: (start, sampled, learned, updated) events
    wall = {"replay": 0.0, "learn": 0.0, "n": 0}  # timing "wall": seconds

    def env_step(record: bool):
        buf.add(new_row)
        for _ in range(utd):
            if timing == "wall":
                torch.cuda.synchronize(dev)
                t0 = time.perf_counter()
                batch, idx, w = buf.sample(batch_size)
                torch.cuda.synchronize(dev)
                t1 = time.perf_counter()
                td = learner.step(batch, w)
                torch.cuda.synchronize(dev)
                t2 = time.perf_counter()
                buf.update_priorities(idx, td)
                torch.cuda.synchronize(dev)
                t3 = time.perf_counter()
                if record:
                    wall["replay"] += (t1 - t0) + (t3 - t2)
                    wall["learn"] += t2 - t1
                    wall["n"] += 1
                continue
            ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)] if record else None
            if record:
                ev[0].record(stream)
            batch, idx, w = buf.sample(batch_size)
            if record:
                ev[1].record(stream)
            td = learner.step(batch, w)
            if record:
                ev[2].record(stream)
            buf.update_priorities(idx, td)
            if record:
                ev[3].record(stream)
                marks.append(ev)

    for _ in range(warmup):
        env_step(False)
    torch.cuda.synchronize(dev)
    total = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    total.record(stream)
    for _ in range(steps):
        env_step(True)
    end.record(stream)
    torch.cuda.synchronize(dev)

    replay = learn = 0.0
    for e0, e1, e2, e3 in marks:
        replay += e0.elapsed_time(e1) + e2.elapsed_time(e3)
        learn += e1.elapsed_time(e2)
    n_grad = len(marks)
    if timing == "wall":
        replay, learn, n_grad = 1e3 * wall["replay"], 1e3 * wall["learn"], wall["n"]
    elapsed = total.elapsed_time(end)
    result = {
        "utd": utd, "batch_size": batch_size, "capacity": capacity, "num_q": num_q,
        "steps": steps, "timing": timing, "replay_ms": replay, "learn_ms": learn,
        "step_ms": elapsed / steps,
        "replay_share": replay / (replay + learn) if replay + learn > 0 else 0.0,
        "replay_us_per_grad_step": 1e3 * replay / max(1, n_grad),
    }
    if hasattr(buf, "status"):
        result["status"] = buf.status()

    if trace:
        from torch.profiler import ProfilerActivity, profile

        with profile(activities=[ProfilerActivity.CPU, ProfilerActivity.CUDA]) as prof:
            for _ in range(3):
                env_step(False)
            torch.cuda.synchronize(dev)
        prof.export_chrome_trace(trace)
        result["trace"] = trace
    return result


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--utd", type=int, default=32)
    ap.add_argument("--batch-size", type=int, default=256)
    ap.add_argument("--capacity", type=int, default=1_000_000)
    ap.add_argument("--obs-dim", type=int, default=32)
    ap.add_argument("--act-dim", type=int, default=8)
    ap.add_argument("--num-q", type=int, default=2, help="critics (10 = REDQ-style)")
    ap.add_argument("--steps", type=int, default=60)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--device", default="cuda")
    ap.add_argument("--trace", default=None, help="Chrome trace output path")
    ap.add_argument("--timing", default="events", choices=["events", "wall"])
    args = ap.parse_args()
    print(json.dumps(run(args.utd, args.batch_size, args.capacity, args.obs_dim, args.act_dim,
                         args.num_q, args.steps, args.warmup, device=args.device,
                         trace=args.trace, timing=args.timing)))


if __name__ == "__main__":
    main()
