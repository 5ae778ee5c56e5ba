"""Test configuration: the `gpu` marker and import paths.

`-m "not gpu"` runs on any host (oracle vs golden vectors, host logic, the
C-ABI library's exports, multi-rank host logic on gloo). `-m gpu` runs the
CUDA engine against the oracle on a B200.
"""

import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "triton-per_b200"), os.path.join(ROOT, "tests", "golden")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")
