"""The C-ABI library loads, exports every declared entry point, and its
ctypes mirror matches the C header's struct layout (CPU only, no launches)."""

import ctypes
import os
import subprocess
import tempfile

import pytest

from per_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_library_exports_every_header_function():
    names = _lib.header_functions()
    assert len(names) >= 8
    for n in names:
        assert hasattr(_lib.lib, n), f"libper_b200.so does not export {n}"
        assert n in _lib.SIGNATURES, f"{n} has no ctypes signature"
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    assert set(names) <= exported


def test_abi_version():
    assert _lib.lib.per_abi_version() == 2  # 2: per_store_t.elem_bytes (16-bit rows)


C_PROBE = r"""
#include <stddef.h>
#include <stdio.h>
#include "per_b200.h"
#define F(T, m) printf(#T "." #m " %zu\n", offsetof(T, m))
int main(void) {
  printf("per_layout_t %zu\nper_store_t %zu\nper_field_t %zu\n",
         sizeof(per_layout_t), sizeof(per_store_t), sizeof(per_field_t));
  F(per_layout_t, level_nodes); F(per_layout_t, level_len); F(per_layout_t, scratch_bytes);
  F(per_store_t, claims); F(per_store_t, level_len); F(per_store_t, num_levels);
  F(per_store_t, capacity); F(per_store_t, storage); F(per_store_t, size_cursor);
  F(per_store_t, scratch_bytes); F(per_store_t, alpha); F(per_store_t, eps);
  F(per_field_t, dim); F(per_field_t, col_offset);
  return 0;
}
"""


def test_ctypes_structs_match_header():
    with tempfile.TemporaryDirectory() as d:
        src = os.path.join(d, "probe.c")
        exe = os.path.join(d, "probe")
        open(src, "w").write(C_PROBE)
        subprocess.run(["gcc", "-I", os.path.join(ROOT, "include"), src, "-o", exe], check=True)
        lines = subprocess.run([exe], capture_output=True, text=True, check=True).stdout.split("\n")
    got = dict(l.rsplit(" ", 1) for l in lines if l)
    py = {"per_layout_t": _lib.Layout, "per_store_t": _lib.Store, "per_field_t": _lib.Field}
    for k, v in got.items():
        if "." in k:
            t, m = k.split(".")
            assert getattr(py[t], m).offset == int(v), k
        else:
            assert ctypes.sizeof(py[k]) == int(v), k


@pytest.mark.parametrize("cap,top,levels", [(1, 1, 3), (1000, 1, 3), (100_000, 1, 3),
                                            (1_000_000, 2, 3), (2_000_000, 2, 3),
                                            (8_000_000, 3, 4), (64_000_000, 3, 4)])
def test_layout(cap, top, levels):
    lay = _lib.layout(cap)
    assert lay.capacity_padded == -(-cap // 1024) * 1024
    assert lay.num_blocks == -(-cap // 1024)
    assert lay.top_level == top and lay.num_levels == levels
    assert lay.level_nodes[top] <= 4096
    for k in range(1, lay.num_levels):
        # every child of every live node is allocated
        assert lay.level_len[k - 1] >= 32 * lay.level_nodes[k]
        assert lay.level_len[k] % 32 == 0
    assert lay.level_len[2] >= lay.num_blocks


def test_layout_rejects_bad_capacity():
    with pytest.raises(_lib.PerError):
        _lib.layout(0)
    with pytest.raises(_lib.PerError):
        _lib.layout((1 << 30) + 1)


def test_entry_points_validate_before_touching_the_gpu():
    L = _lib.lib
    assert L.per_sample_fused(None, None, 1, 0.4, None, 1, None, None, None) == 2
    assert L.per_update_priorities(None, None, None, 1, None) == 2
    assert L.per_add(None, None, 0, 0, None) == 2
    assert L.per_rebuild_sums(None, None) == 2
    bad = _lib.Store()
    bad.capacity = 1000
    assert L.per_rebuild_sums(ctypes.byref(bad), None) == 1  # num_levels/top mismatch
    assert L.per_error_string(3) == b"empty input"


def test_no_cpu_fallback():
    from per_b200 import PERBuffer
    with pytest.raises(RuntimeError, match="CUDA"):
        PERBuffer(100, {"x": 1}, device="cpu")
