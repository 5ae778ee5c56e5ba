"""Launch modes of the grid-synchronising kernels (B200).

The sample kernel (max exchange between CTAs) and the grid path of the
update are launched with a programmatic dependency by default, eagerly and in
graphs; PER_COOPERATIVE=1 launches them cooperatively outside stream capture.
Both modes must give identical results: a child process with the variable
set samples and updates the same store from the same uniforms and writes its
outputs, which must equal this process's bit for bit."""

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
    rows = {{"x": rng.standard_normal((cap, 6), dtype=np.float32)}}
    buf = make_buffer(cap, {{"x": 6}}, rows, cases.leaves_abs_normal(rng, cap))
    out = []
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


def test_cooperative_and_default_launches_agree(tmp_path):
    script = tmp_path / "child.py"
    script.write_text(CHILD.format(tests=HERE))
    res = {}
    for mode in ("0", "1"):
        env = dict(os.environ, PER_COOPERATIVE=mode)
        path = tmp_path / f"out_{mode}.npz"
        subprocess.run([sys.executable, str(script), str(path)], env=env, check=True,
                       timeout=300)
        with np.load(path) as z:
            res[mode] = [z[k] for k in sorted(z.files, key=lambda s: int(s.split("_")[1]))]
    assert len(res["0"]) == len(res["1"]) == 7
    for a, b in zip(res["0"], res["1"]):
        np.testing.assert_array_equal(a, b)
