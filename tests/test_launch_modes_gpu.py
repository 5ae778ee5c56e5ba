"""Launch and gather modes of the sample and update kernels (B200).

The sample kernel (max exchange between CTAs) and the grid path of the
update are launched with a programmatic dependency by default, eagerly and in
graphs; PER_COOPERATIVE=1 launches them cooperatively outside stream capture.
Rows move by four-row tensor gathers by default; PER_GATHER4=0 moves them by
one bulk copy per row (many rows per SM) or cp.async chains (a few). Every
mode must give identical results: a child process per mode samples and
updates the same store from the same uniforms (batches 256 and 65,536, rows
of 6 and 74 floats) and writes its outputs, which must agree bit for bit."""

import os
import subprocess
import sys

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))

CHILD = r"""
import os, sys, numpy as np, torch
for p in ({tests!r}, os.path.join({tests!r}, "golden"), os.path.dirname({tests!r}),
          os.path.join(os.path.dirname({tests!r}), "triton-per_b200")):
    sys.path.insert(0, p)
import cases
from helpers import make_buffer
def run():
    rng = np.random.default_rng(11)
    cap = 400_000
    out = []
    for width in (6, 74):
        rows = {{"x": rng.standard_normal((cap, width), dtype=np.float32)}}
        buf = make_buffer(cap, {{"x": width}}, rows, cases.leaves_abs_normal(rng, cap))
        for batch in (256, 65536):
            rand = torch.from_numpy(rng.random(batch, dtype=np.float32)).cuda()
            views, idx, w = buf.sample_from_uniforms(rand, 0.5)
            out += [views["x"].cpu().numpy(), idx.cpu().numpy(), w.cpu().numpy()]
            td = torch.from_numpy(rng.standard_normal(batch).astype(np.float32)).cuda()
            buf.update_priorities(idx, td)  # 65,536 entries: the grid path
        out.append(buf.priorities.cpu().numpy())
        torch.cuda.synchronize()
        assert all(v == 0 for k, v in buf.status().items()
                   if k in ("errors", "timeouts")), buf.status()
    return out
if __name__ == "__main__":
    np.savez(sys.argv[1], *run())
"""


MODES = {
    "default": {},
    "cooperative": {"PER_COOPERATIVE": "1"},
    "no_gather4": {"PER_GATHER4": "0"},
}


def test_launch_and_gather_modes_agree(tmp_path):
    script = tmp_path / "child.py"
    script.write_text(CHILD.format(tests=HERE))
    res = {}
    for mode, extra in MODES.items():
        env = {k: v for k, v in os.environ.items() if k not in ("PER_COOPERATIVE", "PER_GATHER4")}
        env.update(extra)
        path = tmp_path / f"out_{mode}.npz"
        subprocess.run([sys.executable, str(script), str(path)], env=env, check=True,
                       timeout=300)
        with np.load(path) as z:
            res[mode] = [z[k] for k in sorted(z.files, key=lambda s: int(s.split("_")[1]))]
    for mode in MODES:
        assert len(res[mode]) == 14
        for a, b in zip(res["default"], res[mode]):
            np.testing.assert_array_equal(a, b)
