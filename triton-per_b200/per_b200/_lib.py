"""ctypes binding of the engine's C ABI (include/per_b200.h).

The structs below mirror per_layout_t, per_store_t and per_field_t field by
field; tests/test_abi.py checks their sizes and offsets against the C header.
The library is the in-tree libper_b200.so built by per_b200.build; there is no
fallback: importing this module without it raises.
"""

from __future__ import annotations

import ctypes
import os
import re

PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG, "libper_b200.so")
HEADER = os.path.join(os.path.dirname(os.path.dirname(PKG)), "include", "per_b200.h")

MAX_LEVELS = 7
STATUS_WORDS = 16
MAX_FIELDS = 16
NOALLOC_MAX_CAPACITY = 1048576
IPC_HANDLE_BYTES = 64

i64 = ctypes.c_int64
u64 = ctypes.c_uint64
i32 = ctypes.c_int32
vp = ctypes.c_void_p

ERRORS = {
    0: "PER_OK", 1: "PER_ERR_INVALID_ARGUMENT", 2: "PER_ERR_NULL_POINTER", 3: "PER_ERR_EMPTY",
    4: "PER_ERR_TOO_LARGE", 5: "PER_ERR_MISALIGNED", 6: "PER_ERR_CUDA", 7: "PER_ERR_NO_DEVICE",
}

STATUS_NAMES = ["errors", "fallbacks", "zero_walks", "clamps", "bad_indices", "timeouts",
                "foreign"]
EVT_BARRIER_TIMEOUT = 0x1
EVT_EMPTY_BUFFER = 0x2
EVT_BAD_INDEX = 0x4
EVT_INCONSISTENT_TREE = 0x8
EVT_PEER_TIMEOUT = 0x10


class Layout(ctypes.Structure):
    _fields_ = [
        ("capacity", i64),
        ("capacity_padded", i64),
        ("num_blocks", i64),
        ("num_levels", i32),
        ("top_level", i32),
        ("level_nodes", i64 * MAX_LEVELS),
        ("level_len", i64 * MAX_LEVELS),
        ("scratch_bytes", i64),
    ]


class Store(ctypes.Structure):
    _fields_ = [
        ("levels", vp * MAX_LEVELS),
        ("claims", vp * MAX_LEVELS),
        ("level_len", i64 * MAX_LEVELS),
        ("num_levels", i32),
        ("top_level", i32),
        ("capacity", i64),
        ("storage", vp),
        ("row_dim", i64),
        ("row_stride", i64),
        ("size_cursor", vp),
        ("max_priority", vp),
        ("status", vp),
        ("scratch", vp),
        ("scratch_bytes", i64),
        ("alpha", ctypes.c_float),
        ("eps", ctypes.c_float),
        ("elem_bytes", i32),
    ]


class Field(ctypes.Structure):
    _fields_ = [
        ("data", vp),
        ("dim", i64),
        ("stride", i64),
        ("col_offset", i64),
    ]


# name -> (restype, argtypes); every function declared in include/per_b200.h
SIGNATURES = {
    "per_layout": (ctypes.c_int, [i64, ctypes.POINTER(Layout)]),
    "per_row_stride": (i64, [i64]),
    "per_sample_fused": (ctypes.c_int, [ctypes.POINTER(Store), vp, i64, ctypes.c_float, vp, i64,
                                        vp, vp, vp]),
    "per_update_priorities": (ctypes.c_int, [ctypes.POINTER(Store), vp, vp, i64, vp]),
    "per_add": (ctypes.c_int, [ctypes.POINTER(Store), ctypes.POINTER(Field), i32, i64, vp]),
    "per_rebuild_sums": (ctypes.c_int, [ctypes.POINTER(Store), vp]),
    "per_update_priorities_noalloc": (ctypes.c_int, [ctypes.POINTER(Store), vp, vp, i64, vp]),
    "per_shard_stats": (ctypes.c_int, [ctypes.POINTER(Store), vp, vp]),
    "per_sample_sharded": (ctypes.c_int, [ctypes.POINTER(Store), i32, i32, i64, vp, vp, i64,
                                          ctypes.c_float, vp, i64, vp, vp, vp, vp, vp, vp]),
    "per_normalize": (ctypes.c_int, [vp, vp, vp, i64, vp]),
    "per_sample_fused_rng": (ctypes.c_int, [ctypes.POINTER(Store), u64, vp, i64, ctypes.c_float, vp,
                                            i64, vp, vp, vp]),
    "per_sample_sharded_rng": (ctypes.c_int, [ctypes.POINTER(Store), i32, i32, i64, vp, u64, vp, i64,
                                              ctypes.c_float, vp, i64, vp, vp, vp, vp, vp, vp]),
    "per_sample_sharded_p2p_rng": (ctypes.c_int, [ctypes.POINTER(Store), i32, i32, i64, vp, u64, vp,
                                                  i64, ctypes.c_float, vp, i64, vp, vp, vp, vp, vp]),
    "per_sample_sharded_p2p_local_rng": (ctypes.c_int, [ctypes.POINTER(Store), i32, i32, i64, vp, u64,
                                                        vp, i64, ctypes.c_float, vp, i64, vp, vp, vp,
                                                        vp, vp]),
    "per_sample_sharded_p2p_max_batch": (ctypes.c_int, [ctypes.POINTER(Store), vp]),
    "per_mailbox_create": (ctypes.c_int, [ctypes.POINTER(vp), vp]),
    "per_mailbox_open": (ctypes.c_int, [vp, ctypes.POINTER(vp)]),
    "per_mailbox_close": (ctypes.c_int, [vp]),
    "per_mailbox_destroy": (ctypes.c_int, [vp]),
    "per_sample_sharded_p2p": (ctypes.c_int, [ctypes.POINTER(Store), i32, i32, i64, vp, vp, i64,
                                              ctypes.c_float, vp, i64, vp, vp, vp, vp, vp]),
    "per_update_priorities_shard": (ctypes.c_int, [ctypes.POINTER(Store), i64, vp, vp, i64, vp]),
    "per_update_priorities_shard_count": (ctypes.c_int, [ctypes.POINTER(Store), i64, vp, vp, i64, vp,
                                                         vp]),
    "per_error_string": (ctypes.c_char_p, [ctypes.c_int]),
    "per_last_cuda_error": (ctypes.c_int, []),
    "per_abi_version": (ctypes.c_int, []),
}


def header_functions(path: str = HEADER) -> list[str]:
    """Names of the functions that include/per_b200.h declares."""
    text = open(path).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return re.findall(r"^\s*(?:int|int64_t|const char\*|void)\s+(per_\w+)\s*\(", text, flags=re.M)


def _load():
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"per_b200: {LIB_PATH} is missing; build it with `python per_b200/build.py` "
            "(nvcc, sm_100a). There is no CPU fallback.")
    lib = ctypes.CDLL(LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


lib = _load()
ABI_VERSION = lib.per_abi_version()


class PerError(RuntimeError):
    """A PER_ERR_* code returned by the engine."""

    def __init__(self, what: str, code: int):
        msg = f"per_b200: {what} failed: {lib.per_error_string(code).decode()} ({ERRORS.get(code, code)})"
        if code == 6:
            msg += f", cudaError {lib.per_last_cuda_error()}"
        super().__init__(msg)
        self.code = code


def check(what: str, rc: int) -> None:
    if rc != 0:
        raise PerError(what, rc)


def layout(capacity: int) -> Layout:
    out = Layout()
    check("per_layout", lib.per_layout(capacity, ctypes.byref(out)))
    return out
