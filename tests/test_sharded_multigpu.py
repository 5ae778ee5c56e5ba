"""Sharded buffer across real GPUs (one process per GPU, NCCL): the union of
the ranks' draws equals one buffer's draw, weights are normalised by the max
over all ranks, routed updates reach their owners; sample() draws the same
in-kernel uniforms on every rank. Both exchanges are run:
NCCL collectives between kernels, and the in-kernel exchange over peer
memory (several calls in a row, so the mailboxes' sequence numbers advance,
and one batch above the one-wave limit, which takes the collective path).
With normalize="rank" the draws and rows are the same and each rank's weights
are the global ones divided by their largest value on that rank.
Skipped with fewer GPUs than ranks."""

import os
import socket
import sys

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))
WORLD = 2


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q, exchange, normalize="global"):
    for p in (os.path.dirname(HERE), os.path.join(os.path.dirname(HERE), "triton-per_b200"), HERE):
        if p not in sys.path:
            sys.path.insert(0, p)
    import datetime

    import torch.distributed as dist

    from per_b200.sharded import ShardedPERBuffer

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        rng = np.random.default_rng(3)
        shard_cap = 50_000
        total = shard_cap * world
        leaves = rng.lognormal(0, 1, total).astype(np.float32)
        rows = rng.standard_normal((total, 6), dtype=np.float32)
        buf = ShardedPERBuffer(total, {"x": 6}, device=f"cuda:{rank}", seed=9, exchange=exchange,
                               normalize=normalize)
        assert buf.exchange == exchange
        lo = rank * shard_cap
        b = buf.shard.buf
        b.add({"x": torch.from_numpy(rows[lo: lo + shard_cap]).cuda()})
        b.priorities[:shard_cap] = torch.from_numpy(leaves[lo: lo + shard_cap]).cuda()
        b.rebuild_sums()
        draws = []
        for k, bs in enumerate((8192, 300, 8192, buf.p2p_max_batch + 4096 if exchange == "p2p" else 0)):
            if bs == 0:
                continue
            rand = np.random.default_rng(4 + k).random(bs, dtype=np.float32)
            res = buf.sample_from_uniforms(torch.from_numpy(rand).cuda(), beta=0.5)
            n = int(res.count.item())
            assert (res.idx[n:] == -1).all()
            draws.append((rand, res.idx[:n].cpu().numpy(), res.w[:n].cpu().numpy(),
                          res.pos[:n].cpu().numpy(), res.views["x"][:n].cpu().numpy()))
        from oracle import oracle

        for bs in (4096, 700):  # sample(): the in-kernel Philox stream, same on every rank
            c0 = int(buf._rng_counter.item())
            res = buf.sample(bs, beta=0.5)
            n = int(res.count.item())
            assert int(buf._rng_counter.item()) == c0 + bs
            draws.append((oracle.philox_uniforms(buf.seed, c0, bs), res.idx[:n].cpu().numpy(),
                          res.w[:n].cpu().numpy(), res.pos[:n].cpu().numpy(),
                          res.views["x"][:n].cpu().numpy()))
        upd_idx = np.random.default_rng(50 + rank).integers(0, total, 2000)
        upd_td = np.random.default_rng(60 + rank).random(2000).astype(np.float32)
        buf.update_priorities(torch.from_numpy(upd_idx), torch.from_numpy(upd_td), route=True)
        torch.cuda.synchronize()
        q.put((rank, draws, upd_idx, upd_td, b.priorities[:shard_cap].cpu().numpy(), leaves, rows,
               b.status()))
        buf.close()
    except Exception as e:
        q.put((rank, repr(e)))
        raise
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("exchange,normalize",
                         [("nccl", "global"), ("p2p", "global"), ("p2p", "rank"), ("nccl", "rank")])
@pytest.mark.skipif(torch.cuda.device_count() < WORLD, reason="needs 2 GPUs")
def test_sharded_across_gpus(exchange, normalize):
    from oracle import oracle

    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, WORLD, port, q, exchange, normalize)) for r in range(WORLD)]
    for p in procs:
        p.start()
    results = [q.get(timeout=300) for _ in range(WORLD)]
    for p in procs:
        p.join(timeout=120)
    errors = [r for r in results if len(r) == 2]
    assert not errors, errors
    assert all(p.exitcode == 0 for p in procs)
    results.sort(key=lambda t: t[0])
    leaves, rows = results[0][5], results[0][6]
    total = leaves.size
    lv = np.zeros(-(-total // 1024) * 1024, np.float32)
    lv[:total] = leaves
    for k in range(len(results[0][1])):
        rand = results[0][1][k][0]
        idx_o, _, csum = oracle.sample(lv, total, total, rand, 0.5)
        idx_g = np.full(rand.size, -1, np.int64)
        w_g = np.zeros(rand.size, np.float32)
        for rank, draws, *_ in results:
            _, idx, w, pos, x = draws[k]
            assert (idx_g[pos] == -1).all()
            idx_g[pos] = idx
            w_g[pos] = w
            np.testing.assert_array_equal(x, rows[idx])
        assert (idx_g >= 0).all()
        _, exc, bad = oracle.classify_indices(idx_g, idx_o, rand, csum, total)
        assert bad.size == 0
        w_o = oracle.weights_for(lv, csum[-1], total, idx_g, 0.5)
        if normalize == "global":
            np.testing.assert_allclose(w_g, w_o, rtol=1e-6)
        else:  # each rank's weights over its own largest one
            for rank, draws, *_ in results:
                pos = draws[k][3]
                if pos.size:
                    assert draws[k][2].max() == 1.0
                    np.testing.assert_allclose(draws[k][2], w_o[pos] / w_o[pos].max(), rtol=2e-6)
    st = oracle.OracleStore(total, {"x": 6})
    st.set_priorities(lv)
    for rank, _, upd_idx, upd_td, *_ in results:
        st.update_priorities(upd_idx, upd_td)
    sc = total // WORLD
    for rank, _, _, _, shard_leaves, *rest in results:
        np.testing.assert_allclose(shard_leaves, st.priorities[rank * sc:(rank + 1) * sc], rtol=1e-6)
        assert rest[-1]["errors"] == 0 and rest[-1]["timeouts"] == 0
