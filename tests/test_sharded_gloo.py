"""Multi-rank host logic of ShardedPERBuffer on gloo (CPU, world size 2).

Each rank drives a CPU shard with the CUDA shard's semantics
(tests/shard_fake.py); the test checks that the exchange of shard totals,
the owner routing, the max all-reduce and the update routing reproduce one
buffer holding every slot (the oracle on the concatenated leaves)."""

import os
import socket
import sys

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

HERE = os.path.dirname(os.path.abspath(__file__))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, cap, q, normalize="global"):
    for p in (os.path.dirname(HERE), os.path.join(os.path.dirname(HERE), "triton-per_b200"), HERE):
        if p not in sys.path:
            sys.path.insert(0, p)
    import torch.distributed as dist

    from oracle import oracle
    from per_b200.sharded import ShardedPERBuffer
    from shard_fake import CpuShard

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime

    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        rng = np.random.default_rng(7)
        fields = {"x": 2}
        shard_cap = -(-cap // world)
        all_leaves = rng.lognormal(0, 1, shard_cap * world).astype(np.float32)
        rows = np.arange(shard_cap * world * 2, dtype=np.float32).reshape(-1, 2)
        shard = CpuShard(shard_cap, fields)
        buf = ShardedPERBuffer(cap, fields, device="cpu", seed=3, shard=shard, normalize=normalize)
        lo = rank * shard_cap
        buf.add({"x": torch.from_numpy(rows[lo: lo + shard_cap])})
        shard.set_leaves(all_leaves[lo: lo + shard_cap])

        # ---- sample: union over ranks == one buffer over all slots
        rand = torch.from_numpy(np.random.default_rng(11).random(4096, dtype=np.float32))
        res = buf.sample_from_uniforms(rand, beta=0.4)
        n = int(res.count.item())
        got = (res.idx[:n].numpy(), res.w[:n].numpy(), res.pos[:n].numpy(),
               res.views["x"][:n].numpy())
        # ---- update with routing: every rank submits entries for both shards
        upd_idx = np.random.default_rng(20 + rank).integers(0, shard_cap * world, 300)
        upd_td = np.random.default_rng(30 + rank).random(300).astype(np.float32) * 3
        buf.update_priorities(torch.from_numpy(upd_idx), torch.from_numpy(upd_td), route=True)
        q.put((rank, got, upd_idx, upd_td, shard.st.priorities[:shard_cap].copy(),
               all_leaves, rows, rand.numpy()))
    except Exception as e:  # report instead of leaving the parent waiting
        q.put((rank, repr(e)))
        raise
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("normalize", ["global", "rank"])
def test_sharded_union_equals_single_buffer(normalize):
    """normalize="rank": the same draws, each rank's weights divided by their
    largest value on that rank (no max all-reduce)."""
    world, cap = 2, 6000
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, cap, q, normalize))
             for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(world)]
    errors = [r for r in results if len(r) == 2]
    assert not errors, errors
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    results.sort(key=lambda t: t[0])
    sys.path.insert(0, os.path.dirname(HERE))
    from oracle import oracle

    _, _, _, _, _, all_leaves, rows, rand = results[0]
    total_cap = all_leaves.size
    lv = np.zeros(-(-total_cap // 1024) * 1024, np.float32)
    lv[:total_cap] = all_leaves
    idx_o, w_o, csum = oracle.sample(lv, total_cap, total_cap, rand, 0.4)
    idx_g = np.full(rand.size, -1, np.int64)
    w_g = np.zeros(rand.size, np.float32)
    for rank, (idx, w, pos, x), *_ in results:
        assert (idx_g[pos] == -1).all(), "a draw was taken by two ranks"
        idx_g[pos] = idx
        w_g[pos] = w
        np.testing.assert_array_equal(x, rows[idx])  # rows come from the owner's shard
    assert (idx_g >= 0).all(), "a draw was taken by no rank"
    eq, exc, bad = oracle.classify_indices(idx_g, idx_o, rand, csum, total_cap)
    assert bad.size == 0 and exc <= 40
    w_ref = oracle.weights_for(lv, csum[-1], total_cap, idx_g, 0.4)
    if normalize == "global":
        np.testing.assert_allclose(w_g, w_ref, rtol=1e-5)
    else:
        for rank, (idx, w, pos, x), *_ in results:
            assert w.max() == 1.0
            np.testing.assert_allclose(w, w_ref[pos] / w_ref[pos].max(), rtol=1e-5)

    # routed update: every shard equals the oracle's update of the whole store
    st = oracle.OracleStore(total_cap, {"x": 2})
    st.set_priorities(lv)
    for rank, _, upd_idx, upd_td, *_ in results:
        st.update_priorities(upd_idx, upd_td)
    shard_cap = total_cap // world
    for rank, _, _, _, shard_leaves, *_ in results:
        np.testing.assert_allclose(shard_leaves, st.priorities[rank * shard_cap:(rank + 1) * shard_cap],
                                   rtol=1e-6)


# ---------------------------------------------------------------- failures
def _failure_worker(rank, world, port, mode, q):
    for p in (os.path.dirname(HERE), os.path.join(os.path.dirname(HERE), "triton-per_b200"), HERE):
        if p not in sys.path:
            sys.path.insert(0, p)
    import datetime

    import torch.distributed as dist

    from per_b200.sharded import ShardedPERBuffer
    from shard_fake import CpuShard

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=10))
    outcome = "ok"
    try:
        cap = 4000 if (mode == "mismatch" and rank == 1) else 6000
        buf = ShardedPERBuffer(cap, {"x": 2}, device="cpu", seed=3,
                               shard=CpuShard(-(-cap // world), {"x": 2}))
        buf.add({"x": torch.zeros(100, 2)})
        if mode == "dead" and rank == 1:
            q.put((rank, "left"))  # this rank leaves between steps, before the collective
            q.close()
            q.join_thread()  # the message is out before the process ends
            os._exit(0)
        buf.sample(64)  # collective: exchanges the shard totals
    except ValueError as e:
        outcome = "ValueError: " + str(e)[:80]
    except RuntimeError as e:  # the process group reports the missing peer
        outcome = "RuntimeError: " + str(e)[:80]
    q.put((rank, outcome))
    try:
        dist.destroy_process_group()
    except Exception:
        pass


@pytest.mark.parametrize("mode", ["mismatch", "dead"])
def test_sharded_failures_surface_as_errors(mode):
    """Host-side failure detection on gloo ranks: ranks that disagree on the
    buffer layout all raise ValueError at construction; a rank that leaves
    between steps makes the survivor's next collective raise (no hang)."""
    world = 2
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_failure_worker, args=(r, world, port, mode, q))
             for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
    if mode == "mismatch":
        assert all(v.startswith("ValueError") for v in results.values()), results
    else:
        assert results[1] == "left"
        assert results[0].startswith("RuntimeError"), results
