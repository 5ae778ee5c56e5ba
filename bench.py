"""Benchmark of the prioritized-replay hot path on B200.

Default workload (N=1): the high-UTD replay loop on 1,000,000 x 74 float32
transitions (fields obs32/action8/reward1/next_obs32/done1, rows ~N(0,1),
done in {0,1}), priorities (|N(0,1)|+1e-6)^0.6: one step = add 1 transition +
32 x (sample batch 256 with beta 0.4 -> update 256 TD errors |N(0,1)|).
Metric: sampled transitions per second (sample + gather + IS weights).

  value     device-resident: the step captured in a CUDA graph, CUDA events
            around exactly K replays after W warm-up replays (max over ranks).
  e2e       the same loop through the public PERBuffer API, eager, with the
            step's inputs copied from pinned host memory and the sampled
            batches (rows, idx, w of every round, sampled into caller-owned
            device slots with sample(..., out=)) copied back to pinned host
            memory at the end of the step, on a second stream that overlaps
            the next step (double-buffered slots; the timed region ends
            after the last read-back).
  roofline  the fused sample kernel alone on the same store: algorithmic
            bytes (8*row_dim + 16 per draw) over its CUDA-event launch time,
            against the measured HBM copy peak.
  sweep     the same kernel over batch 32..65,536 on heavy-tailed
            priorities (lognormal(0,2), 1% exact zeros).
  cpu_baseline  the oracle (CPU restatement of the reference's torch
            backend, C, all host threads) on a bounded sample of the same loop.
  cpu_baseline_sumtree  the reference's own CPU baseline, its float64
            SumTree (baselines/cpu_sumtree.py) restated in C (one thread, as
            the reference's per-draw host loop), on this loop and on the
            100,000-slot CPU configuration, plus the plain-Python restatement
            (the reference's own code path) on the latter.
  parity    one 65,536-draw sample of the timed store checked against the
            oracle: indices equal except excused float32 prefix ties (counted).
  sharded64m  the sharded configuration (64,000,000 x 74, global batch
            65,536, strong scaling) on the same N GPUs.

--impl reference times that CPU implementation alone on the same loop.

N>1 (torchrun, one rank per GPU): the same loop weak-scaled over the sharded
buffer: each rank holds a 1,000,000 x 74 shard (N x 1M slots in all), a step
is add 1 per rank + 32 x (sharded sample of a global batch of N x 256 ->
update of each rank's own draws); every sample exchanges the shard totals
(all-gather) and the max weight (all-reduce) over NCCL. value = all ranks'
transitions / max step time over ranks.

--workload sharded64m: 64,000,000 x 74 slots split over the N ranks
(lognormal(0,1) priorities), one step = sharded sample of a global batch of
65,536 -> update of each rank's draws (strong scaling).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
for _p in (ROOT, os.path.join(ROOT, "triton-per_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import numpy as np  # noqa: E402
import torch  # noqa: E402

FIELDS_74 = {"obs": 32, "action": 8, "reward": 1, "next_obs": 32, "done": 1}
CAPACITY = 1_000_000
ROW_DIM = 74
BATCH = 256
ROUNDS = 32
BETA = 0.4
SWEEP = [32, 128, 512, 2048, 8192, 32768, 65536]
# beyond the configured sweep: several tiles per warp (more than one wave)
SWEEP_LARGE = [131072, 262144]
METRIC = "sampled transitions/s (sample+gather+IS)"
UNIT = "transitions/s"


def algo_bytes(batch: int, row_dim: int) -> int:
    """Algorithmic bytes of one fused sample: row read + row write + idx + w + uniform."""
    return batch * (8 * row_dim + 16)


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


# ---------------------------------------------------------------- clocks
class ClockSampler:
    """SM clock and clock-event (throttle) reasons of one GPU while the timed
    region runs: NVML polled every 2 ms, else `nvidia-smi -lms 100` (reads
    only; nothing is set)."""

    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown"}
    SMI_FIELDS = ("clocks.sm,clocks.max.sm,clocks_event_reasons.active")

    def __init__(self, cuda_index: int):
        self.cuda_index = cuda_index
        self.samples: list[tuple[float, int]] = []
        self.max_mhz = None
        self.source = "unavailable"
        self.error = None
        self._stop = threading.Event()
        self._t = None
        self._nvml = None
        self._smi = None

    def _nvml_handle(self, nv):
        """The NVML device behind torch's cuda:<index> (UUID match, else the
        CUDA_VISIBLE_DEVICES entry, else the same index)."""
        try:
            want = str(torch.cuda.get_device_properties(self.cuda_index).uuid).lower()
            want = want.removeprefix("gpu-")
            for i in range(nv.nvmlDeviceGetCount()):
                h = nv.nvmlDeviceGetHandleByIndex(i)
                u = nv.nvmlDeviceGetUUID(h)
                u = (u.decode() if isinstance(u, bytes) else u).lower().removeprefix("gpu-")
                if u == want:
                    return h, i
        except Exception:
            pass
        vis = [v.strip() for v in os.environ.get("CUDA_VISIBLE_DEVICES", "").split(",") if v.strip()]
        if self.cuda_index < len(vis):
            v = vis[self.cuda_index]
            if v.isdigit():
                return nv.nvmlDeviceGetHandleByIndex(int(v)), int(v)
            return nv.nvmlDeviceGetHandleByUUID(v), None
        return nv.nvmlDeviceGetHandleByIndex(self.cuda_index), self.cuda_index

    def __enter__(self):
        try:
            import pynvml

            pynvml.nvmlInit()
            h, self._index = self._nvml_handle(pynvml)
            self._nvml, self._h = pynvml, h
            self.max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM))
            self.source = "nvml"
            self._t = threading.Thread(target=self._poll, daemon=True)
            self._t.start()
        except Exception as e:  # no NVML: nvidia-smi in the background
            self.error = repr(e)[:200]
            self._nvml = None
            self._start_smi()
        return self

    def _start_smi(self):
        import subprocess

        idx = self.cuda_index
        vis = [v.strip() for v in os.environ.get("CUDA_VISIBLE_DEVICES", "").split(",") if v.strip()]
        if idx < len(vis):
            idx = vis[idx]
        try:
            self._smi = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.SMI_FIELDS}", "--format=csv,noheader,nounits",
                 "-i", str(idx), "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.source = "nvidia-smi"
        except OSError as e:
            self.error = repr(e)[:200]

    def _poll(self):
        nv, h = self._nvml, self._h
        get_reasons = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons",
                              getattr(nv, "nvmlDeviceGetCurrentClocksThrottleReasons", None))
        while not self._stop.is_set():
            try:
                mhz = float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM))
                bits = int(get_reasons(h)) if get_reasons else 0
                self.samples.append((mhz, bits))
            except Exception as e:
                self.error = repr(e)[:200]
            self._stop.wait(0.002)

    def __exit__(self, *exc):
        self._stop.set()
        if self._t:
            self._t.join(timeout=2)
        if self._smi is not None:
            self._smi.terminate()
            try:
                out, _ = self._smi.communicate(timeout=5)
            except Exception:
                self._smi.kill()
                out = ""
            for line in (out or "").splitlines():
                parts = [p.strip() for p in line.split(",")]
                try:
                    mhz, mx, bits = float(parts[0]), float(parts[1]), int(parts[2], 16)
                except (ValueError, IndexError):
                    continue
                self.max_mhz = mx
                self.samples.append((mhz, bits))

    def summary(self):
        out = {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [],
               "samples": len(self.samples), "source": self.source}
        if self.error and not self.samples:
            out["error"] = self.error
        if not self.samples:
            return out
        reasons = set()
        for _, bits in self.samples:
            for b, name in self.REASONS.items():
                if bits & b:
                    reasons.add(name)
        out["sm_mhz"] = statistics.median(m for m, _ in self.samples)
        out["reasons"] = sorted(reasons)
        return out


# ---------------------------------------------------------------- distributed
def dist_setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    elif torch.cuda.is_available():
        torch.cuda.set_device(local)
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([x], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([x], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


# ---------------------------------------------------------------- workload
def make_store(device, seed, priorities="absnormal", storage_dtype=torch.float32):
    from per_b200 import PERBuffer

    buf = PERBuffer(CAPACITY, FIELDS_74, device=device, storage_dtype=storage_dtype)
    g = torch.Generator(device=device).manual_seed(seed)
    chunk = 250_000
    for s in range(0, CAPACITY, chunk):
        n = min(chunk, CAPACITY - s)
        batch = {k: torch.randn(n, d, generator=g, device=device)
                 for k, d in FIELDS_74.items() if k != "done"}
        batch["done"] = (torch.rand(n, 1, generator=g, device=device) < 0.5).float()
        buf.add(batch)
    if priorities == "absnormal":
        leaves = (torch.randn(CAPACITY, generator=g, device=device).abs() + 1e-6) ** 0.6
    else:  # heavy-tailed with 1% exact zeros
        leaves = torch.empty(CAPACITY, device=device).log_normal_(0.0, 2.0, generator=g)
        zeros = torch.randperm(CAPACITY, generator=g, device=device)[: CAPACITY // 100]
        leaves[zeros] = 0.0
    buf.priorities[:CAPACITY] = leaves
    buf.rebuild_sums()
    torch.cuda.synchronize()
    return buf


def make_wide_store(device, seed=11, capacity=2_000_000, row_dim=4096):
    """2M x 4096 float32 rows ~U(0,1) (32 GB, image-feature-like), priorities
    (|N(0,1)| + 1e-6)^0.6: the wide-row gather configuration."""
    from per_b200 import PERBuffer

    buf = PERBuffer(capacity, {"feat": row_dim}, device=device)
    g = torch.Generator(device=device).manual_seed(seed)
    chunk = 100_000
    for s0 in range(0, capacity, chunk):
        n = min(chunk, capacity - s0)
        buf.add({"feat": torch.rand(n, row_dim, generator=g, device=device)})
    leaves = (torch.randn(capacity, generator=g, device=device).abs() + 1e-6) ** 0.6
    buf.priorities[:capacity] = leaves
    buf.rebuild_sums()
    torch.cuda.synchronize()
    return buf


def utd_step(buf, row, td):
    """One step of the high-UTD loop: add 1, then 32 x (sample 256 -> update 256)."""
    buf.add(row)
    for r in range(ROUNDS):
        _, idx, _ = buf.sample(BATCH, BETA)
        buf.update_priorities(idx, td[r])


def packed_rows(views):
    """The [batch, row_dim] rows behind a sample's field views (they are column
    slices of one packed output, first field first): no copy, no kernel."""
    v0 = next(iter(views.values()))
    return v0.as_strided((v0.shape[0], ROW_DIM), (v0.stride(0), 1))


def capture(fn, warm=3, generators=()):
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(warm):
            fn()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    for gen in generators:
        g.register_generator_state(gen)
    with torch.cuda.graph(g):
        fn()
    torch.cuda.synchronize()
    return g


def time_replays(g, iters, world):
    st = torch.cuda.current_stream()
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    barrier(world)
    torch.cuda.synchronize()
    torch.cuda.nvtx.range_push("timed")  # the launch list (ncu --nvtx-include timed/)
    a.record(st)
    for _ in range(iters):
        g.replay()
    b.record(st)
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    barrier(world)
    return a.elapsed_time(b)  # ms


def kernel_time_us(buf, batch, reps=20, launches=16, beta=BETA):
    """Average CUDA-event time of one fused-sample launch (graph of `launches`).
    Uniforms are drawn inside the kernel from the buffer's advancing stream,
    so every launch of every replay gathers new rows: a replayed set of fixed
    uniforms would gather the same rows each time, which then come from L2
    instead of HBM for batches whose rows fit in it."""

    def fn():
        for _ in range(launches):
            buf.sample(batch, beta)

    g = capture(fn, warm=2)
    for _ in range(3):
        g.replay()
    ms = time_replays(g, reps, 1)
    return ms * 1000.0 / (reps * launches)


def update_time_us(buf, n, reps=20, launches=16, seed=8):
    g0 = torch.Generator(device=buf.device).manual_seed(seed)
    idxs = [torch.randint(0, CAPACITY, (n,), generator=g0, device=buf.device) for _ in range(launches)]
    tds = [torch.randn(n, generator=g0, device=buf.device).abs() for _ in range(launches)]

    def fn():
        for i, t in zip(idxs, tds):
            buf.update_priorities(i, t)

    g = capture(fn, warm=2)
    for _ in range(3):
        g.replay()
    ms = time_replays(g, reps, 1)
    return ms * 1000.0 / (reps * launches)


def e2e_loop(buf, steps, warmup, world, seed=9):
    """Public API, eager, host buffers: H2D of the step's inputs (the added
    transition, the TD errors of all rounds) from pinned memory; every round
    samples into its slot of a device block through sample(..., out=) and
    updates; the step ends with the D2H of every sampled batch (rows, idx, w
    of all rounds: three copies) into pinned memory, on a copy stream that
    overlaps the next step's sampling (which uses the other block)."""
    dev = buf.device
    g = np.random.default_rng(seed)
    h_row = {k: torch.from_numpy(g.standard_normal((1, d), dtype=np.float32)).pin_memory()
             for k, d in FIELDS_74.items()}
    h_td = torch.from_numpy(np.abs(g.standard_normal((ROUNDS, BATCH))).astype(np.float32)).pin_memory()
    # two sets of device slots and host buffers: step k's read-back (on its
    # own stream) overlaps step k+1's sampling, which uses the other set
    sets = []
    for _ in range(2):
        d_rows = torch.empty(ROUNDS, BATCH, ROW_DIM, device=dev)
        d_idx = torch.empty(ROUNDS, BATCH, dtype=torch.int64, device=dev)
        d_w = torch.empty(ROUNDS, BATCH, device=dev)
        sets.append({
            "dev": (d_rows, d_idx, d_w),
            "host": (torch.empty(ROUNDS, BATCH, ROW_DIM).pin_memory(),
                     torch.empty(ROUNDS, BATCH, dtype=torch.int64).pin_memory(),
                     torch.empty(ROUNDS, BATCH).pin_memory()),
            "outs": [buf.sample_out(BATCH, rows=d_rows[r], idx=d_idx[r], w=d_w[r])
                     for r in range(ROUNDS)],
            "copied": None,
        })
    h2d = sum(v.numel() * 4 for v in h_row.values()) + h_td.numel() * 4
    d2h = ROUNDS * BATCH * (ROW_DIM * 4 + 8 + 4)
    st = torch.cuda.current_stream()
    cs = torch.cuda.Stream(device=dev)
    k = [0]

    def step():
        s = sets[k[0] % 2]
        k[0] += 1
        if s["copied"] is not None:  # its previous read-back has left the slots
            st.wait_event(s["copied"])
        row = {kk: v.to(dev, non_blocking=True) for kk, v in h_row.items()}
        tds = h_td.to(dev, non_blocking=True).unbind(0)
        buf.add(row)
        for r in range(ROUNDS):
            _, idx, _ = buf.sample(BATCH, BETA, out=s["outs"][r])
            buf.update_priorities(idx, tds[r])
        cs.wait_stream(st)
        with torch.cuda.stream(cs):
            for h, d in zip(s["host"], s["dev"]):
                h.copy_(d, non_blocking=True)
            s["copied"] = torch.cuda.Event()
            s["copied"].record(cs)

    for _ in range(warmup):
        step()
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    barrier(world)
    torch.cuda.synchronize()
    a.record(st)
    for _ in range(steps):
        step()
    st.wait_stream(cs)  # every read-back of the timed steps is inside the region
    b.record(st)
    torch.cuda.synchronize()
    barrier(world)
    ms = max_over_ranks(a.elapsed_time(b), world)
    return ms / steps, h2d, d2h


# ---------------------------------------------------------------- sharded
def make_sharded(device, rank, world, total_capacity, priorities, seed=1, exchange="auto",
                 normalize="global"):
    from per_b200.sharded import ShardedPERBuffer

    sb = ShardedPERBuffer(total_capacity, FIELDS_74, device=device, seed=seed, exchange=exchange,
                          normalize=normalize)
    cap = sb.shard_capacity
    buf = sb.shard.buf
    g = torch.Generator(device=device).manual_seed(1000 + rank)
    chunk = 1_000_000
    for s0 in range(0, cap, chunk):
        n = min(chunk, cap - s0)
        batch = {k: torch.randn(n, d, generator=g, device=device)
                 for k, d in FIELDS_74.items() if k != "done"}
        batch["done"] = (torch.rand(n, 1, generator=g, device=device) < 0.5).float()
        buf.add(batch)
    if priorities == "absnormal":
        leaves = (torch.randn(cap, generator=g, device=device).abs() + 1e-6) ** 0.6
    else:
        leaves = torch.empty(cap, device=device).log_normal_(0.0, 1.0, generator=g)
    buf.priorities[:cap] = leaves
    buf.rebuild_sums()
    torch.cuda.synchronize()
    return sb


def sharded_utd_step(sb, row, td, world):
    sb.add(row)
    for r in range(ROUNDS):
        res = sb.sample(BATCH * world, BETA)
        sb.update_priorities(res.idx, td[r])


def sharded64m_step(sb, td, batch):
    res = sb.sample(batch, BETA)
    sb.update_priorities(res.idx, td)


def time_eager(fn, iters, world):
    st = torch.cuda.current_stream()
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    barrier(world)
    torch.cuda.synchronize()
    a.record(st)
    for _ in range(iters):
        fn()
    b.record(st)
    torch.cuda.synchronize()
    barrier(world)
    return a.elapsed_time(b)


def sharded_e2e(sb, gb, rounds, steps, warmup, world, with_add):
    """The sharded step through the public API, eager, host buffers both
    ways: H2D of the step's TD errors (and added row), each round sampled into
    its slot of a device block with sample(..., out=) (in-kernel exchange) and
    updated, then every slot (rows, idx, w) back to pinned host memory on a
    copy stream that overlaps the next step (double-buffered blocks)."""
    dev = sb.device
    h_td = torch.abs(torch.randn(rounds, gb)).pin_memory()
    h_row = {k: torch.randn(1, d).pin_memory() for k, d in FIELDS_74.items()}
    p2p = sb.exchange == "p2p" and gb <= sb.p2p_max_batch
    sets = []
    for _ in range(2):
        d_rows = torch.empty(rounds, gb, ROW_DIM, device=dev)
        outs = [sb.sample_out(gb, rows=d_rows[r]) for r in range(rounds)] if p2p else None
        sets.append({"rows": d_rows, "outs": outs, "copied": None,
                     "h_rows": torch.empty(rounds, gb, ROW_DIM).pin_memory(),
                     "h_idx": torch.empty(rounds, gb, dtype=torch.int64).pin_memory(),
                     "h_w": torch.empty(rounds, gb).pin_memory()})
    st = torch.cuda.current_stream()
    cs = torch.cuda.Stream(device=dev)
    k = [0]

    def step():
        s_ = sets[k[0] % 2]
        k[0] += 1
        if s_["copied"] is not None:
            st.wait_event(s_["copied"])
        tdd = h_td.to(dev, non_blocking=True)
        if with_add:
            sb.add({kk: v.to(dev, non_blocking=True) for kk, v in h_row.items()})
        results = []
        for r in range(rounds):
            res = sb.sample(gb, BETA, out=s_["outs"][r]) if p2p else sb.sample(gb, BETA)
            sb.update_priorities(res.idx, tdd[r])
            results.append(res)
        cs.wait_stream(st)
        with torch.cuda.stream(cs):
            for r, res in enumerate(results):
                if not p2p:
                    s_["h_rows"][r].copy_(packed_rows(res.views), non_blocking=True)
                s_["h_idx"][r].copy_(res.idx, non_blocking=True)
                s_["h_w"][r].copy_(res.w, non_blocking=True)
            if p2p:
                s_["h_rows"].copy_(s_["rows"], non_blocking=True)
            s_["copied"] = torch.cuda.Event()
            s_["copied"].record(cs)

    for _ in range(warmup):
        step()
    n = max(3, min(steps, 20))
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    barrier(world)
    torch.cuda.synchronize()
    a.record(st)
    for _ in range(n):
        step()
    st.wait_stream(cs)
    b.record(st)
    torch.cuda.synchronize()
    barrier(world)
    e_ms = max_over_ranks(a.elapsed_time(b), world) / n
    return e_ms, h_td.numel() * 4 + (ROW_DIM * 4 if with_add else 0), rounds * gb * (ROW_DIM * 4 + 12)


def sharded_measure(args, world, rank, local, big, normalize="global"):
    """The sharded buffer across the ranks (collective; rank 0 gets the dict).

    normalize="rank": weights divided by each rank's own max (no max exchange).

    big: 64,000,000 x 74 slots split over the ranks (lognormal(0,1)
    priorities), one step = sample of a global batch of 65,536 -> update of
    each rank's own draws (strong scaling). Otherwise the weak-scaling UTD
    loop: 1,000,000 x 74 slots per rank, add 1 per rank + 32 x (sample of
    256 x N -> update)."""
    dev = torch.device("cuda", local)
    total_cap = 64_000_000 if big else CAPACITY * world
    sb = make_sharded(dev, rank, world, total_cap, "lognormal" if big else "absnormal",
                      exchange=args.exchange, normalize=normalize)
    g = torch.Generator(device=dev).manual_seed(100 + rank)
    gb = 65_536 if big else BATCH * world
    rounds = 1 if big else ROUNDS
    td = torch.randn(ROUNDS, gb, generator=g, device=dev).abs()
    row = {k: torch.randn(1, d, generator=g, device=dev) for k, d in FIELDS_74.items()}
    p2p = sb.exchange == "p2p" and gb <= sb.p2p_max_batch
    # kernels per sample+update (uniforms drawn inside the sample kernel): in-kernel
    # exchange -> sample, update; collectives -> stats, sample, normalise, update
    # (+ NCCL all-gather and all-reduce)
    per_round = 2 if p2p else 4
    if big:
        fn = lambda: sharded64m_step(sb, td[0], gb)  # noqa: E731
        launches = per_round
    else:
        fn = lambda: sharded_utd_step(sb, row, td, world)  # noqa: E731
        launches = 1 + ROUNDS * per_round
    per_step = gb * rounds
    if normalize == "rank":
        exchange_desc = ("shard totals exchanged inside the sample kernel over NVLink peer "
                         "memory (CUDA IPC mailboxes); weights over each rank's own max"
                         if p2p else "NCCL all-gather of shard totals per sample; weights "
                         "over each rank's own max")
    else:
        exchange_desc = ("shard totals and max weight exchanged inside the sample kernel over "
                         "NVLink peer memory (CUDA IPC mailboxes)" if p2p else
                         "NCCL all-gather of shard totals + all-reduce max per sample")
    for _ in range(max(args.warmup, 3)):
        fn()
    torch.cuda.synchronize()
    # capture the step (kernels and NCCL collectives) into a CUDA graph; every
    # rank must have captured before any rank replays, else all run eagerly
    graph = None
    try:
        graph = capture(fn, warm=0)
        ok = 1.0
    except Exception as e:  # capture unsupported here: time the eager loop
        graph = None
        ok = 0.0
        if rank == 0:
            print(f"# graph capture failed, timing eagerly: {e!r}"[:300], file=sys.stderr)
    ok = -max_over_ranks(-ok, world)  # min over ranks
    if ok < 1.0:
        graph = None
    if graph is not None:
        for _ in range(max(args.warmup, 3)):
            graph.replay()
        torch.cuda.synchronize()
        mode = "CUDA graph of one step" + ("" if p2p else " (kernels + NCCL collectives)")
        with ClockSampler(local) as clk:
            ms = time_replays(graph, args.steps, world)
    else:
        mode = "eager (host-driven)"
        with ClockSampler(local) as clk:
            ms = time_eager(fn, args.steps, world)
    graph = None  # release graphs holding NCCL calls before the group is destroyed
    ms = max_over_ranks(ms, world)
    ms_per_step = ms / args.steps
    value = per_step / (ms_per_step / 1e3)
    st = sb.shard.buf.status()
    bad = max_over_ranks(float(st["errors"] or st["timeouts"]), world)
    if bad:
        raise SystemExit(f"device status reports errors: {st}")
    e_ms, h2d, d2h = sharded_e2e(sb, gb, rounds, args.steps, 2, world, with_add=not big)
    sb.close()
    out = None
    if rank == 0:
        out = {
            "value": value, "ms_per_step": ms_per_step,
            "scaling": "strong" if big else "weak",
            "workload": ("sharded-64Mx74: sample 65536 beta 0.4 -> update own draws"
                         if big else
                         "sharded utd 1Mx74 per rank: add 1 + 32 x (sample 256/rank beta 0.4 "
                         "-> update own draws)"),
            "capacity_total": total_cap, "shard_capacity": sb.shard_capacity,
            "row_dim": ROW_DIM, "global_batch": gb, "rounds": rounds,
            "parallelism": f"sharded x{world} ({exchange_desc})",
            "l2": "rows (320 MB per 1M slots) exceed L2",
            "timing": mode + ", CUDA events, max over ranks",
            "gpu_launches": launches * args.steps,
            "clocks": clk.summary(),
            "e2e": {"value": per_step / (e_ms / 1e3), "unit": UNIT,
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
        }
    del sb
    torch.cuda.empty_cache()
    return out


def run_sharded(args, world, rank, local):
    """N>1 (or --workload sharded64m): the sharded buffer across the ranks.
    The line carries the weak-scaling UTD loop (N>1) and the 64M strong
    configuration (`sharded64m`), or the latter alone with --workload."""
    big_only = args.workload == "sharded64m"
    main_ = sharded_measure(args, world, rank, local, big=big_only)
    big = main_ if big_only else sharded_measure(args, world, rank, local, big=True)
    # the opt-in rank-local normalisation, reported beside the exact global one
    rank_norm = None
    if world > 1 and not args.no_rank_norm:
        rank_norm = (sharded_measure(args, world, rank, local, big=big_only, normalize="rank"),
                     None if big_only else
                     sharded_measure(args, world, rank, local, big=True, normalize="rank"))
    if rank == 0:
        line = {
            "metric": METRIC, "value": main_["value"], "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": main_["ms_per_step"],
            "higher_is_better": True, "scaling": main_["scaling"], "vs_baseline": None,
            "dtype": "f32", "data": "synthetic",
            "config": {k: main_[k] for k in ("workload", "capacity_total", "shard_capacity",
                                             "row_dim", "global_batch", "rounds", "parallelism",
                                             "l2", "timing")},
            "gpu_launches": main_["gpu_launches"],
            "clocks": main_["clocks"],
            "e2e": main_["e2e"],
            "sharded64m": {k: big[k] for k in ("value", "ms_per_step", "e2e", "parallelism",
                                               "timing", "global_batch", "capacity_total")},
        }
        if rank_norm is not None:
            keys = ("value", "ms_per_step", "e2e", "parallelism")
            line["rank_normalized"] = {
                "weights": "each rank's weights divided by that rank's largest weight "
                           "(ShardedPERBuffer(normalize='rank')); draws and rows unchanged",
                **{k: rank_norm[0][k] for k in keys}}
            if rank_norm[1] is not None:
                line["rank_normalized"]["sharded64m"] = {k: rank_norm[1][k] for k in keys}
        print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- CPU side
def cpu_loop(seconds=None, steps=None, warmup=0, threads=None):
    """The oracle (reference torch-backend algorithm, C) on the same loop.

    Returns (transitions/s, steps timed, threads)."""
    from oracle import oracle

    threads = threads or os.cpu_count() or 1
    rng = np.random.default_rng(3)
    cap = CAPACITY
    nb = -(-cap // 1024)
    leaves = np.zeros(nb * 1024, np.float32)
    leaves[:cap] = np.power(np.abs(rng.standard_normal(cap)).astype(np.float32) + np.float32(1e-6),
                            np.float32(0.6))
    storage = rng.standard_normal((cap, ROW_DIM), dtype=np.float32)
    bsums = oracle.block_sums(leaves)
    st = oracle.OracleStore.__new__(oracle.OracleStore)
    st.capacity, st.alpha, st.eps, st.row_dim = cap, 0.6, 1e-6, ROW_DIM
    st.num_blocks, st.capacity_padded = nb, nb * 1024
    st.priorities, st.block_sums, st.storage = leaves, bsums, storage
    st.max_priority, st.size, st.cursor = np.float32(1.0), cap, 0
    st._offsets = {"row": (0, ROW_DIM)}
    st.fields = {"row": ROW_DIM}
    row = rng.standard_normal((1, ROW_DIM), dtype=np.float32)
    td = np.abs(rng.standard_normal((ROUNDS, BATCH))).astype(np.float32)
    csum = np.empty(cap, np.float32)

    def one_step():
        st.add({"row": row})
        for r in range(ROUNDS):
            rand = rng.random(BATCH, dtype=np.float32)
            oracle.lib().oracle_cumsum(st.priorities, cap, csum, threads)
            idx, w, _ = oracle.sample_from_csum(st.priorities, csum, cap, st.size, rand, BETA, threads)
            _ = st.storage[idx]  # gather
            st.update_priorities(idx, td[r])

    for _ in range(warmup):
        one_step()
    t0 = time.perf_counter()
    n = 0
    while True:
        one_step()
        n += 1
        el = time.perf_counter() - t0
        if steps is not None and n >= steps:
            break
        if seconds is not None and el >= seconds:
            break
    return ROUNDS * BATCH * n / el, n, threads


def sumtree_loop(config: int, seconds: float, impl: str = "c"):
    """The reference's CPU sum tree (oracle/sumtree.py) on a bounded sample.

    config 0: 100,000 x 74 slots, rounds of sample 256 (beta 0.4) -> gather
    -> update 256 |N(0,1)| TD errors with ~10% duplicate indices.
    config 1: 1,000,000 x 74 slots, steps of add 1 + 32 x (sample 256 ->
    gather -> update 256). impl "c": the C restatement; "python": the plain
    Python restatement (the reference's own loops). One host thread.
    Returns (transitions/s, rounds timed)."""
    from oracle import sumtree

    rng = np.random.default_rng(4 + config)
    cap = 100_000 if config == 0 else CAPACITY
    leaves = np.power(np.abs(rng.standard_normal(cap)) + 1e-6, 0.6)
    if impl == "c":
        st = sumtree.SumTreeStore(cap, ROW_DIM)
        st.build_from_leaves(leaves)
    else:
        st = sumtree.PySumTree(cap, ROW_DIM)
        st.tree[cap:] = leaves
        for k in range(cap - 1, 0, -1):  # set-up, untimed
            st.tree[k] = st.tree[2 * k] + st.tree[2 * k + 1]
    st.storage[:] = rng.standard_normal((cap, ROW_DIM), dtype=np.float32)
    st.size = cap
    row = rng.standard_normal((1, ROW_DIM), dtype=np.float32)
    td = np.abs(rng.standard_normal((ROUNDS, BATCH))).astype(np.float32)

    def one_round(r):
        idx, w = st.sample_from_uniforms(rng.random(BATCH), BETA)[:2]
        if impl == "c":
            st.gather(idx)
        upd = idx.copy()
        k = BATCH // 10  # ~10% duplicates of other entries of the batch
        upd[rng.choice(BATCH, k, replace=False)] = upd[rng.integers(0, BATCH, k)]
        st.update_priorities(upd, td[r % ROUNDS])

    def one_step():
        if config == 1:
            if impl == "c":
                st.add(row)
            for r in range(ROUNDS):
                one_round(r)
        else:
            one_round(0)

    one_step()  # warm-up
    rounds_per_step = ROUNDS if config == 1 else 1
    t0 = time.perf_counter()
    n = 0
    while True:
        one_step()
        n += rounds_per_step
        el = time.perf_counter() - t0
        if el >= seconds:
            break
    return BATCH * n / el, n


def cpu_sumtree_baseline(seconds: float):
    """cpu_baseline_sumtree of the bench line (see the module docstring)."""
    v1, n1 = sumtree_loop(1, seconds, "c")
    v0, n0 = sumtree_loop(0, seconds / 2, "c")
    p0, m0 = sumtree_loop(0, seconds / 2, "python")
    return {
        "value": v1, "unit": UNIT, "cores": 1, "host_cores": os.cpu_count(), "threads": 1,
        "kind": "port",
        "impl": "the reference's float64 SumTree (baselines/cpu_sumtree.py) restated in C, "
                "one draw and one index at a time on one host thread",
        "sample": f"{n1} sample 256 + update 256 rounds of this loop (1M x 74, add 1 per 32 rounds)",
        "config0_100Kx74": {"value": v0, "rounds": n0,
                            "python_loop_value": p0, "python_loop_rounds": m0,
                            "workload": "sample 256 beta 0.4 -> update 256, ~10% duplicate indices"},
    }


def parity_check(buf, batch=65536, seed=21):
    """One `batch`-draw sample of the store checked against the oracle: the
    excused float32 prefix ties are counted; any other index mismatch fails
    the run. Test-side checker (the oracle is not timed)."""
    from oracle import oracle

    g = torch.Generator(device=buf.device).manual_seed(seed)
    rand = torch.rand(batch, generator=g, device=buf.device)
    _, idx, _ = buf.sample_from_uniforms(rand, BETA)
    torch.cuda.synchronize()
    size = int(buf._size_cursor[0].item())
    lv = buf.priorities.cpu().numpy()
    rnp = rand.cpu().numpy()
    idx_o, _, csum = oracle.sample(lv, buf.capacity, size, rnp, BETA, nthreads=os.cpu_count() or 1)
    eq, excused, bad = oracle.classify_indices(idx.cpu().numpy(), idx_o, rnp, csum, size)
    if bad.size:
        raise SystemExit(f"parity: {bad.size} index mismatches outside float32 ties")
    return {"draws": batch, "equal": eq, "excused_ties": excused, "mismatches": 0,
            "store": "the timed 1M x 74 store after the loop", "checker": "oracle (C)"}


class HostPriorityBuffer:
    """PERBuffer API over priorities kept and searched on the host: the
    reference's CPU baselines restated under oracle/ (checker code, used
    here only as the comparison arms of the replay-share profile). Rows live
    on the GPU and are gathered there, as in the reference's CpuSumTreePER
    (cpu_sumtree.py:41-97): each sample walks the host structure and sends the
    indices and weights over PCIe; each update brings the TD errors back.

    kind "cpu_sumtree": the float64 SumTree (C restatement, one draw at a
    time); kind "torch_cpu": the reference torch backend's algorithm (C
    restatement: full cumsum of the priorities per sample, all host threads)."""

    def __init__(self, capacity, fields, device, kind):
        from oracle import oracle, sumtree

        self.kind = kind
        self.capacity = capacity
        self.device = torch.device(device)
        self.fields = dict(fields)
        self._offsets, o = {}, 0
        for name, d in fields.items():
            self._offsets[name] = (o, o + d)
            o += d
        self.storage = torch.zeros(capacity, o, device=self.device)
        self.cursor = 0
        self.size = 0
        self._rng = np.random.default_rng(0)
        self._oracle = oracle
        self._threads = os.cpu_count() or 1
        if kind == "cpu_sumtree":
            self.st = sumtree.SumTreeStore(capacity, 1)
        else:
            self.st = oracle.OracleStore(capacity, {"x": 1})

    def add(self, batch):
        n = next(iter(batch.values())).shape[0]
        idx = (torch.arange(n, device=self.device) + self.cursor) % self.capacity
        for name, (a, b) in self._offsets.items():
            self.storage[idx, a:b] = batch[name].reshape(n, -1).to(self.storage.dtype)
        if self.kind == "cpu_sumtree":
            self.st.add(np.zeros((n, 1), np.float32))
        else:
            self.st.add({"x": np.zeros((n, 1), np.float32)})
        self.cursor = (self.cursor + n) % self.capacity
        self.size = min(self.size + n, self.capacity)

    def sample(self, batch_size, beta=0.4):
        if self.kind == "cpu_sumtree":
            idx, w = self.st.sample_from_uniforms(self._rng.random(batch_size), beta)
        else:
            idx, w, _ = self._oracle.sample(self.st.priorities, self.capacity, self.size,
                                            self._rng.random(batch_size, dtype=np.float32), beta,
                                            nthreads=self._threads)
        idx_t = torch.from_numpy(idx).to(self.device)
        out = self.storage[idx_t]
        views = {name: out[:, a:b] for name, (a, b) in self._offsets.items()}
        return views, idx_t, torch.from_numpy(w).to(self.device)

    def update_priorities(self, indices, td_errors):
        self.st.update_priorities(indices.cpu().numpy(),
                                  td_errors.detach().reshape(-1).abs().cpu().numpy())


def replay_share_arms(steps=20):
    """The UTD replay-share profile (per_b200.profile_utd: SAC-style learner,
    2 critics, UTD 32, batch 256, 1M slots) with this engine and with the
    reference's two CPU baselines as the replay backend, every arm timed the
    reference's way (host clock around synchronised phases); the engine also
    by CUDA events (device timeline, nothing synchronised)."""
    from per_b200 import profile_utd

    fields = {"obs": 32, "action": 8, "reward": 1, "next_obs": 32, "done": 1}
    keep = ("replay_share", "replay_us_per_grad_step", "learn_ms", "replay_ms", "step_ms", "timing")
    out = {}
    r = profile_utd.run(steps=steps, warmup=3, timing="events")
    out["b200_events"] = {k: r[k] for k in keep}
    r = profile_utd.run(steps=steps, warmup=3, timing="wall")
    out["b200_wall"] = {k: r[k] for k in keep}
    for kind, n in (("cpu_sumtree", max(2, steps // 4)), ("torch_cpu", max(2, steps // 4))):
        buf = HostPriorityBuffer(1_000_000, fields, "cuda", kind)
        r = profile_utd.run(steps=n, warmup=1, timing="wall", buffer=buf)
        out[kind] = {k: r[k] for k in keep}
        del buf
    out["config"] = "utd 32, batch 256, 1M slots (200k filled), 2 critics, SAC-style update"
    return out


# ---------------------------------------------------------------- main
def traffic_from_profiles(key: str):
    """DRAM bytes per launch (dram__bytes_read.sum + dram__bytes_write.sum of
    one ncu capture) from profiles/traffic.json, or None."""
    try:
        with open(os.path.join(ROOT, "profiles", "traffic.json")) as f:
            v = json.load(f).get(key)
        return int(v) if v is not None else None
    except (OSError, ValueError):
        return None


def run_reference(args, world, rank):
    if rank != 0:
        return
    v, n, threads = cpu_loop(steps=max(1, args.steps), warmup=args.warmup)
    line = {
        "impl": "reference", "metric": METRIC, "value": v, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ROUNDS * BATCH / v * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic",
        "config": {"workload": "utd-1Mx74: add 1 + 32 x (sample 256 beta 0.4 -> update 256)",
                   "capacity": CAPACITY, "row_dim": ROW_DIM, "batch": BATCH, "rounds": ROUNDS,
                   "parallelism": "host threads"},
        "cpu_baseline": {"value": v, "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": f"{n} full steps ({n * ROUNDS} sample+update rounds) of the loop, "
                                   "oracle restatement of the reference torch backend in C"},
        "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        # the reference's other CPU baseline (its float64 SumTree), same loop
        "cpu_baseline_sumtree": cpu_sumtree_baseline(4.0),
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-seconds", type=float, default=8.0)
    ap.add_argument("--no-sweep", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-share", action="store_true",
                    help="skip the replay-share profile of the N=1 line")
    ap.add_argument("--no-sharded", action="store_true",
                    help="skip the sharded 64M x 74 configuration of the N=1 line")
    ap.add_argument("--no-rank-norm", action="store_true",
                    help="N>1: skip the rank-normalised sharded measurements")
    ap.add_argument("--workload", default="utd", choices=["utd", "sharded64m"])
    ap.add_argument("--exchange", default="auto", choices=["auto", "p2p", "nccl"],
                    help="sharded mode: in-kernel peer-memory exchange or NCCL collectives")
    ap.add_argument("--kernel-only", type=int, default=0, metavar="BATCH",
                    help="profiling aid: eager fused samples of this batch (then updates of 256) "
                         "on the 1M x 74 store, no timing output")
    ap.add_argument("--wide-rows", type=int, default=0, metavar="CAPACITY",
                    help="with --kernel-only: a CAPACITY x 4096 store of the wide-row "
                         "configuration instead (profiling aid; the bench uses 2M rows)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    if args.kernel_only:
        dev = torch.device("cuda", 0)
        torch.cuda.set_device(dev)
        buf = make_wide_store(dev, capacity=args.wide_rows) if args.wide_rows else make_store(dev, seed=1)
        beta = 0.6 if args.wide_rows else BETA
        g = torch.Generator(device=dev).manual_seed(2)
        for _ in range(args.warmup + args.steps):
            r = torch.rand(args.kernel_only, generator=g, device=dev)
            _, idx, _ = buf.sample_from_uniforms(r, beta)
            buf.update_priorities(idx[:BATCH], torch.rand(min(BATCH, idx.numel()), device=dev))
        torch.cuda.synchronize()
        st = buf.status()
        print(json.dumps({"kernel_only": args.kernel_only, "status": st}))
        return

    if args.impl == "reference":
        world = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        run_reference(args, world, rank)
        return

    world, rank, local = dist_setup(args)
    if world > 1 or args.workload == "sharded64m":
        run_sharded(args, world, rank, local)
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()
        return
    dev = torch.device("cuda", local)
    buf = make_store(dev, seed=1 + rank)
    g = torch.Generator(device=dev).manual_seed(100 + rank)
    td = torch.randn(ROUNDS, BATCH, generator=g, device=dev).abs()
    row = {k: torch.randn(1, d, generator=g, device=dev) for k, d in FIELDS_74.items()}

    graph = capture(lambda: utd_step(buf, row, td))
    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        ms = time_replays(graph, args.steps, world)
    ms = max_over_ranks(ms, world)
    ms_per_step = ms / args.steps
    total = ROUNDS * BATCH * world
    value = total / (ms_per_step / 1e3)
    st = buf.status()
    if st["errors"] or st["timeouts"]:
        raise SystemExit(f"device status reports errors: {st}")

    # kernel-level: fused sample at the loop's batch, update at the loop's size
    peak, peak_kind = peaks()
    k_us = kernel_time_us(buf, BATCH)
    u_us = update_time_us(buf, BATCH)
    ab = algo_bytes(BATCH, ROW_DIM)
    achieved = ab / (k_us * 1e-6) / 1e9
    roofline = {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                "frac": achieved / peak, "traffic": traffic_from_profiles("sample_1Mx74_b256"),
                "peak_source": peak_kind, "kernel": "per_sample_kernel_r112 (fused sample, 112-register build)",
                "kernel_us": k_us, "algo_bytes_per_launch": ab, "batch": BATCH,
                "timing": "CUDA events over graph replays of back-to-back launches, uniforms drawn "
                          "in the kernel (new rows every launch)"}
    # the same kernel at the large-batch end of the sweep (1M x 74, batch 65,536)
    k64 = kernel_time_us(buf, 65536, reps=10, launches=8)
    ab64 = algo_bytes(65536, ROW_DIM)
    a64 = ab64 / (k64 * 1e-6) / 1e9
    roofline_large = {"bound": "hbm", "achieved": a64, "peak": peak, "unit": "GB/s",
                      "frac": a64 / peak, "peak_source": peak_kind, "kernel": "per_sample_kernel_r112 (fused sample, 112-register build)",
                      "traffic": traffic_from_profiles("sample_1Mx74_b65536"),
                      "kernel_us": k64, "algo_bytes_per_launch": ab64, "batch": 65536}

    sweep = None
    if not args.no_sweep and rank == 0:
        graph = None
        heavy = make_store(dev, seed=5, priorities="heavy")
        sweep = []
        for b in SWEEP + SWEEP_LARGE:
            us = kernel_time_us(heavy, b, reps=10, launches=8)
            gbs = algo_bytes(b, ROW_DIM) / (us * 1e-6) / 1e9
            sweep.append({"batch": b, "us": round(us, 3), "gbs": round(gbs, 1),
                          "frac": round(gbs / peak, 4),
                          "samples_per_s": round(b / (us * 1e-6))})
        storm = update_time_us(heavy, 65536, reps=5, launches=4)
        sweep.append({"update_storm_65536_us": round(storm, 2)})
        del heavy
        torch.cuda.empty_cache()
        # the same store with 16-bit (bfloat16) rows: half the gather bytes;
        # GB/s counts the 16-bit row bytes (4 * row_dim + 16 per draw)
        heavy16 = make_store(dev, seed=5, priorities="heavy", storage_dtype=torch.bfloat16)
        for b in (8192, 65536, 262144):
            us = kernel_time_us(heavy16, b, reps=10, launches=8)
            gbs = b * (4 * ROW_DIM + 16) / (us * 1e-6) / 1e9
            sweep.append({"batch_bf16_rows": b, "us": round(us, 3), "gbs": round(gbs, 1),
                          "frac": round(gbs / peak, 4), "samples_per_s": round(b / (us * 1e-6))})
        del heavy16
        torch.cuda.empty_cache()
        # wide rows: 2M x 4096 (32 GB), batch 1024, beta 0.6 (sample kernel +
        # whole-GPU row gather kernel per call)
        wide = make_wide_store(dev)
        wus = kernel_time_us(wide, 1024, reps=10, launches=8, beta=0.6)
        wgbs = algo_bytes(1024, 4096) / (wus * 1e-6) / 1e9
        sweep.append({"wide_rows_2Mx4096_batch1024_us": round(wus, 3), "gbs": round(wgbs, 1),
                      "frac": round(wgbs / peak, 4), "samples_per_s": round(1024 / (wus * 1e-6))})
        del wide
        torch.cuda.empty_cache()

    e2e = None
    if not args.no_e2e:
        e_ms, h2d, d2h = e2e_loop(buf, steps=max(5, min(args.steps, 50)), warmup=3, world=world)
        e2e = {"value": ROUNDS * BATCH * world / (e_ms / 1e3), "unit": UNIT,
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h}

    # the CPU legs (host cores; the oracle and the reference's sum tree are
    # timed here, and the oracle checks one large sample of the timed store)
    cpu = cpu_st = parity = share = None
    if rank == 0 and world == 1 and not args.no_cpu:
        v, n, threads = cpu_loop(seconds=args.cpu_seconds, warmup=1)
        cpu = {"value": v, "unit": UNIT, "cores": threads, "kind": "port",
               "sample": f"{n} steps ({n * ROUNDS} sample 256 + update 256 rounds) of the same "
                         "loop, oracle (reference torch-backend algorithm) in C"}
        cpu_st = cpu_sumtree_baseline(args.cpu_seconds / 2)
        parity = parity_check(buf)
        if not args.no_share:
            share = replay_share_arms()

    sh64 = None
    if not args.no_sharded:
        del buf
        graph = None
        torch.cuda.empty_cache()
        big = sharded_measure(args, world, rank, local, big=True)
        if rank == 0:
            sh64 = {k: big[k] for k in ("value", "ms_per_step", "e2e", "parallelism", "timing",
                                        "global_batch", "capacity_total")}

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "utd-1Mx74: add 1 + 32 x (sample 256 beta 0.4 -> update 256)",
                       "capacity": CAPACITY, "row_dim": ROW_DIM, "batch": BATCH,
                       "rounds": ROUNDS, "parallelism": "replicas" if world > 1 else "single",
                       "l2": "storage 296 MB > 126 MB L2 (tree 4 MB stays resident)",
                       "timing": "CUDA graph of one step, CUDA events, max over ranks"},
            "update_us": u_us,
            "roofline": roofline, "roofline_batch65536": roofline_large,
            "sweep": sweep,
            "e2e": e2e,
            "cpu_baseline": cpu,
            "cpu_baseline_sumtree": cpu_st,
            "parity": parity,
            "utd_replay_share": share,
            "sharded64m": sh64,
            "gpu_launches": (1 + 2 * ROUNDS) * args.steps,
            "clocks": clk.summary(),
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist

        graph = None
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
