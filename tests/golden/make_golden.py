"""Generate the golden fixtures by running the REFERENCE itself.

Runs triton-per's own `PERBuffer(..., backend="torch", device="cpu")`
(src/triton_per/buffer.py) and its CPU sum tree `CpuSumTreePER(device="cpu")`
(src/triton_per/baselines/cpu_sumtree.py) on the seeded inputs of cases.py and
stores their outputs as .npz files beside this script. Only runs where the
reference source tree is available (pass the path of its src/ directory or
set TRITON_PER_SRC):

    python tests/golden/make_golden.py <reference>/src

torch runs single-threaded here so that duplicate-index assignments keep the
last occurrence deterministically (with several threads, torch's CPU index_put
splits the index list across threads and the survivor is unspecified).
The sample fixtures call the buffer's `_sample_torch(rand, beta)` with the
stored uniforms and normalise `w / w.max()` exactly as `sample()` does
(buffer.py:92), so that the uniforms are shared with the engine under test.
The sum-tree fixture runs the reference's sample() unchanged except that its
random source (np.random.random, cpu_sumtree.py:77) returns the case's stored
uniforms for the duration of the call, so that the restatement under test can
be fed the same draws.
"""

from __future__ import annotations

import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
import cases  # noqa: E402


def reference_buffer_cls(src):
    sys.path.insert(0, src)
    from triton_per.buffer import BLOCK_P, PERBuffer  # noqa: E402
    return PERBuffer, BLOCK_P


def set_leaves(buf, leaves, BLOCK_P):
    buf.priorities.zero_()
    buf.priorities[: leaves.size] = torch.from_numpy(leaves)
    buf.block_sums[:] = buf.priorities.view(buf.num_blocks, BLOCK_P).sum(dim=1)


def sample_case(PERBuffer, BLOCK_P, name, c):
    buf = PERBuffer(c["capacity"], c["fields"], device="cpu", backend="torch")
    n = next(iter(c["rows"].values())).shape[0]
    buf.add({k: torch.from_numpy(v) for k, v in c["rows"].items()})
    assert buf.size == c["size"] == n
    set_leaves(buf, c["leaves"], BLOCK_P)
    rand = torch.from_numpy(c["rand"])
    idx, w, out = buf._sample_torch(rand, c["beta"])
    w = w / w.max()
    res = dict(idx=idx.numpy(), w=w.numpy(), out_digest=np.array(cases.digest(out.numpy())),
               inputs_digest=np.array(cases.sample_inputs_digest(c)),
               total=np.float32(torch.cumsum(buf.priorities[: buf.capacity], 0)[-1].item()))
    if name == "config1":
        upd_idx = cases.dup_indices(c["dup_rng"], idx.numpy(), c["dup_frac"])
        buf.update_priorities(torch.from_numpy(upd_idx), torch.from_numpy(c["td"]))
        uniq = np.unique(upd_idx)
        res.update(upd_idx=upd_idx, upd_uniq=uniq, upd_leaves=buf.priorities[uniq].numpy(),
                   upd_block_sums=buf.block_sums.numpy().copy(),
                   upd_max_priority=np.float32(buf._max_priority.item()))
        idx2, w2, _ = buf._sample_torch(torch.from_numpy(c["rand2"]), c["beta"])
        res.update(idx2=idx2.numpy(), w2=(w2 / w2.max()).numpy())
    return res


def update_case(PERBuffer, BLOCK_P, c):
    buf = PERBuffer(c["capacity"], {"x": 1}, device="cpu", alpha=c["alpha"], eps=c["eps"],
                    backend="torch")
    set_leaves(buf, c["leaves"], BLOCK_P)
    buf.update_priorities(torch.from_numpy(c["idx"]), torch.from_numpy(c["td"]))
    return dict(leaves=buf.priorities.numpy().copy(), block_sums=buf.block_sums.numpy().copy(),
                max_priority=np.float32(buf._max_priority.item()),
                inputs_digest=np.array(cases.digest(c["leaves"], c["idx"], c["td"])))


def add_case(PERBuffer, BLOCK_P, c):
    buf = PERBuffer(c["capacity"], c["fields"], device="cpu", backend="torch")
    out = {}
    steps = [("add", c["adds"][0]), ("upd", None), ("add", c["adds"][1]), ("add", c["adds"][2])]
    for k, (kind, rows) in enumerate(steps):
        if kind == "add":
            buf.add({"x": torch.from_numpy(rows)})
        else:
            buf.update_priorities(torch.from_numpy(c["upd_idx"]), torch.from_numpy(c["upd_td"]))
        out[f"s{k}_storage"] = buf.storage.numpy().copy()
        out[f"s{k}_leaves"] = buf.priorities.numpy().copy()
        out[f"s{k}_block_sums"] = buf.block_sums.numpy().copy()
        out[f"s{k}_cursor_size"] = np.array([buf._cursor, buf.size], np.int64)
        out[f"s{k}_max_priority"] = np.float32(buf._max_priority.item())
    out["inputs_digest"] = np.array(cases.digest(*c["adds"], c["upd_idx"], c["upd_td"]))
    return out


def sumtree_case(src, c):
    from triton_per.baselines.cpu_sumtree import CpuSumTreePER

    buf = CpuSumTreePER(c["capacity"], c["fields"], device="cpu")
    out = {}
    for k in range(2):
        buf.add({"x": torch.from_numpy(c["adds"][k])})
        out[f"s{k}_tree_after_add"] = buf.tree.tree.copy()
        buf.update_priorities(torch.from_numpy(c["upd_idx"][k]), torch.from_numpy(c["upd_td"][k]))
        out[f"s{k}_tree"] = buf.tree.tree.copy()
        out[f"s{k}_max_priority"] = np.float64(buf._max_priority)
        out[f"s{k}_cursor_size"] = np.array([buf._cursor, buf.size], np.int64)
        rand = c["rand"][k]
        orig = np.random.random
        np.random.random = lambda n, _r=rand: _r[:n].copy()
        try:
            views, idx, w = buf.sample(rand.size, c["beta"])
        finally:
            np.random.random = orig
        out[f"s{k}_idx"] = idx.numpy()
        out[f"s{k}_w"] = w.numpy()
        out[f"s{k}_rows"] = views["x"].numpy().copy()
    out["inputs_digest"] = np.array(cases.sumtree_inputs_digest(c))
    return out


def main():
    src = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("TRITON_PER_SRC")
    if not src:
        raise SystemExit("usage: make_golden.py <path to the reference's src/ directory>")
    torch.set_num_threads(1)
    PERBuffer, BLOCK_P = reference_buffer_cls(src)
    for name, fn in cases.SAMPLE_CASES.items():
        np.savez(os.path.join(HERE, f"sample_{name}.npz"), **sample_case(PERBuffer, BLOCK_P, name, fn()))
    np.savez(os.path.join(HERE, "update_dups.npz"), **update_case(PERBuffer, BLOCK_P, cases.case_update_dups()))
    np.savez(os.path.join(HERE, "update_storm.npz"), **update_case(PERBuffer, BLOCK_P, cases.case_update_storm()))
    np.savez(os.path.join(HERE, "add_wrap.npz"), **add_case(PERBuffer, BLOCK_P, cases.case_add_wrap()))
    np.savez(os.path.join(HERE, "sumtree_small.npz"), **sumtree_case(src, cases.case_sumtree()))
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
