"""Sharded-mode kernels on one B200: several shards emulated in one process.

Each shard is a CUDA store holding a contiguous slice of the global slots. The
shards' statistics are assembled as the all-gather would assemble them, every
shard samples the same global uniforms, the max weight is reduced over the
shards, and the union of the shards' draws must equal the oracle's draw from
one buffer holding every slot (indices up to float32 prefix ties, rows
bit-exact, weights within 1e-6). Updates with global indices must touch only
the owner's slots."""

import ctypes

import numpy as np
import pytest
import torch

import cases
from helpers import SUM_RTOL, check_tree, make_buffer
from oracle import oracle
from per_b200 import _lib
from per_b200.sharded import CudaShard

pytestmark = pytest.mark.gpu


def _shards(world, shard_cap, fields, rows, leaves, sizes):
    shards = []
    for g in range(world):
        sh = CudaShard(shard_cap, fields, torch.device("cuda"), 0.6, 1e-6)
        lo = g * shard_cap
        n = sizes[g]
        if n:
            sh.buf.add({k: torch.from_numpy(v[lo: lo + n]).cuda() for k, v in rows.items()})
        lv = np.zeros(sh.buf.capacity_padded, np.float32)
        lv[:n] = leaves[lo: lo + n]
        sh.buf.priorities.copy_(torch.from_numpy(lv))
        sh.buf.rebuild_sums()
        shards.append(sh)
    return shards


def _sample_all(shards, rand, beta):
    world = len(shards)
    stats = torch.zeros(world, 2, dtype=torch.float64, device="cuda")
    for g, sh in enumerate(shards):
        sh.stats(stats[g])
    res = [sh.sample(g, world, g * sh.buf.capacity, stats, rand, beta) for g, sh in enumerate(shards)]
    gmax = torch.stack([r[5] for r in res]).max().reshape(1)
    for sh, r in zip(shards, res):
        sh.normalize(r[2], r[4], gmax)
    torch.cuda.synchronize()
    return res


@pytest.mark.parametrize("world,shard_cap,full,wide", [(3, 40_000, True, False),
                                                       (4, 5_000, False, False),
                                                       (2, 300_000, True, False),
                                                       (2, 3_000, False, True)])
def test_union_of_shards_equals_one_buffer(world, shard_cap, full, wide):
    rng = np.random.default_rng(world * 7 + shard_cap)
    total = world * shard_cap
    da, db = (2600, 3) if wide else (5, 3)  # wide: rows copied by the separate gather kernel
    fields = {"a": da, "b": db}
    rows = {"a": rng.standard_normal((total, da), dtype=np.float32),
            "b": rng.standard_normal((total, db), dtype=np.float32)}
    leaves = rng.lognormal(0.0, 1.5, total).astype(np.float32)
    sizes = [shard_cap] * world
    if not full:  # partially filled last shard, and one shard without any mass
        sizes[-1] = shard_cap // 3
        leaves[(world - 1) * shard_cap + sizes[-1]:] = 0.0
        leaves[shard_cap: 2 * shard_cap] = 0.0
    shards = _shards(world, shard_cap, fields, rows, leaves, sizes)
    # the single buffer: slots of every shard side by side (unfilled slots hold 0)
    glob_leaves = np.zeros(-(-total // 1024) * 1024, np.float32)
    glob_leaves[:total] = leaves
    packed = np.concatenate([rows["a"], rows["b"]], axis=1)
    n_global = sum(sizes)
    B = 20_000
    rand_np = rng.random(B, dtype=np.float32)
    res = _sample_all(shards, torch.from_numpy(rand_np).cuda(), 0.4)

    idx_g = np.full(B, -1, np.int64)
    w_g = np.zeros(B, np.float32)
    for g, (out, idx, w, pos, count, _) in enumerate(res):
        n = int(count.item())
        p = pos[:n].cpu().numpy()
        assert (idx_g[p] == -1).all(), "a draw was taken by two shards"
        ig = idx[:n].cpu().numpy()
        assert ((ig >= g * shard_cap) & (ig < g * shard_cap + sizes[g])).all()
        idx_g[p] = ig
        w_g[p] = w[:n].cpu().numpy()
        np.testing.assert_array_equal(out[:n].cpu().numpy(), packed[ig])
    assert (idx_g >= 0).all(), "a draw was taken by no shard"

    # oracle: one buffer over all slots (size = all slots when every shard is
    # full; otherwise the clamp of the single buffer does not apply, so only
    # full stores are compared index by index)
    idx_o, w_o, csum = oracle.sample(glob_leaves, total, total, rand_np, 0.4)
    eq, exc, bad = oracle.classify_indices(idx_g, idx_o, rand_np, csum, total)
    print(f"SHARDED world={world} cap={shard_cap}: equal {eq} excused {exc}")
    assert bad.size == 0, f"{bad.size} mismatches outside float32 ties"
    # weights: the oracle's formula with the global size and total on the shards' indices
    w_ref = oracle.weights_for(glob_leaves, csum[-1], n_global, idx_g, 0.4)
    np.testing.assert_allclose(w_g, w_ref, rtol=1e-6, atol=0)
    for sh in shards:
        assert sh.buf.status()["errors"] == 0


def test_update_with_global_indices_touches_only_owned_slots():
    rng = np.random.default_rng(5)
    world, shard_cap = 3, 30_000
    total = world * shard_cap
    leaves = cases.leaves_abs_normal(rng, total)
    rows = {"x": np.zeros((total, 1), np.float32)}
    shards = _shards(world, shard_cap, {"x": 1}, rows, leaves, [shard_cap] * world)
    n = 5000  # grid path
    idx = rng.integers(-1, total, n)  # includes -1 padding
    idx = np.concatenate([idx, idx[:1000]])  # duplicates
    td = (rng.standard_normal(idx.size) * 2).astype(np.float32)
    for g, sh in enumerate(shards):
        sh.update(g * shard_cap, torch.from_numpy(idx).cuda(), torch.from_numpy(td).cuda())
    torch.cuda.synchronize()
    st = oracle.OracleStore(total, {"x": 1})
    lv = np.zeros(st.capacity_padded, np.float32)
    lv[:total] = leaves
    st.set_priorities(lv)
    keep = idx >= 0
    st.update_priorities(idx[keep], td[keep])
    for g, sh in enumerate(shards):
        got = sh.buf.priorities[:shard_cap].cpu().numpy()
        np.testing.assert_allclose(got, st.priorities[g * shard_cap:(g + 1) * shard_cap],
                                   rtol=1e-6, atol=0)
        check_tree(sh.buf)
        s = sh.buf.status()
        own = ((idx >= g * shard_cap) & (idx < (g + 1) * shard_cap)).sum()
        assert s["foreign"] == idx.size - own and s["bad_indices"] == 0


def test_single_rank_p2p_exchange_equals_single_buffer():
    """World 1 through the in-kernel exchange (the rank's own mailbox): the
    draws, rows and weights equal PERBuffer.sample_from_uniforms bit for bit,
    over several calls in a row and past the one-wave limit (collective path)."""
    from per_b200.sharded import ShardedPERBuffer

    rng = np.random.default_rng(17)
    cap = 120_000
    leaves = rng.lognormal(0.0, 1.0, cap).astype(np.float32)
    rows = rng.standard_normal((cap, 7), dtype=np.float32)
    ref = make_buffer(cap, {"x": 7}, {"x": rows}, leaves)
    sb = ShardedPERBuffer(cap, {"x": 7}, device="cuda", exchange="p2p")
    assert sb.exchange == "p2p" and sb.p2p_max_batch >= 148 * 32
    sb.shard.buf.add({"x": torch.from_numpy(rows).cuda()})
    sb.shard.buf.priorities[:cap] = torch.from_numpy(leaves).cuda()
    sb.shard.buf.rebuild_sums()
    for k, bs in enumerate((4096, 33, 65_536, sb.p2p_max_batch, sb.p2p_max_batch + 1)):
        rand = torch.from_numpy(rng.random(bs, dtype=np.float32)).cuda()
        views, idx, w = ref.sample_from_uniforms(rand, 0.4)
        res = sb.sample_from_uniforms(rand, 0.4)
        assert int(res.count.item()) == bs
        assert torch.equal(torch.sort(res.pos.long()).values, torch.arange(bs, device="cuda"))
        order = torch.argsort(res.pos.long())
        assert torch.equal(res.idx[order], idx), k
        assert torch.equal(res.w[order], w), k
        assert torch.equal(res.views["x"][order], views["x"]), k
    st = sb.shard.buf.status()
    assert st["errors"] == 0 and st["timeouts"] == 0
    sb.close()


def test_peer_that_never_publishes_times_out_with_a_status_flag():
    """The in-kernel exchange against a peer mailbox that nothing ever writes
    (a zeroed device buffer standing in for rank 1): every wait gives up after
    its time limit (about a second), the kernel flags PER_EVT_PEER_TIMEOUT and
    counts the timeouts, returns, and the context stays usable."""
    rng = np.random.default_rng(23)
    cap = 50_000
    buf = make_buffer(cap, {"x": 3}, {"x": rng.standard_normal((cap, 3), dtype=np.float32)},
                      rng.lognormal(0.0, 1.0, cap).astype(np.float32))
    mine = ctypes.c_void_p()
    handle = (ctypes.c_char * _lib.IPC_HANDLE_BYTES)()
    assert _lib.lib.per_mailbox_create(ctypes.byref(mine), handle) == 0
    silent = torch.zeros(4096, dtype=torch.uint8, device="cuda")  # never written
    boxes = torch.tensor([mine.value, silent.data_ptr()], dtype=torch.int64, device="cuda")
    b = 64
    rand = torch.rand(b, device="cuda")
    out = torch.empty(b, 3, device="cuda")
    idx = torch.empty(b, dtype=torch.int64, device="cuda")
    w = torch.empty(b, device="cuda")
    pos = torch.empty(b, dtype=torch.int32, device="cuda")
    count = torch.empty(1, dtype=torch.int64, device="cuda")
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = _lib.lib.per_sample_sharded_p2p(buf._store_ref, 0, 2, 0, boxes.data_ptr(), rand.data_ptr(),
                                         b, 0.4, out.data_ptr(), 3, idx.data_ptr(), w.data_ptr(),
                                         pos.data_ptr(), count.data_ptr(), stream)
    assert rc == 0
    torch.cuda.synchronize()
    st = buf.status()
    assert st["errors"] & 0x10, st  # PER_EVT_PEER_TIMEOUT
    assert st["timeouts"] >= 2, st   # the statistics wait and the max wait
    # the context is still usable: an ordinary sample afterwards
    buf.clear_status()
    views, i2, w2 = buf.sample(256, 0.4)
    torch.cuda.synchronize()
    assert buf.status()["errors"] == 0 and (i2 >= 0).all()
    assert _lib.lib.per_mailbox_destroy(mine) == 0
