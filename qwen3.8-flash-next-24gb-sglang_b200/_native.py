"""ctypes binding of ``lib/libw2a16_moe.so`` (the C ABI of ``include/w2a16_moe.h``).

The library is required: importing the ops without it raises immediately. There is no Python or
CPU fallback for any kernel; a missing library or a non-CUDA tensor is an error.
"""
from __future__ import annotations

import ctypes
import os
import threading

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "lib", "libw2a16_moe.so")

# path choice of w2a16_moe_decode_layer_slots_ex (include/w2a16_moe.h)
PATH_AUTO, PATH_PER_TOKEN, PATH_BATCHED = 0, 1, 2
BATCHED_AUTO_TOKENS = 64

STATUS = {
    0: "ok", 1: "unsupported shape", 2: "misaligned stride or base address", 3: "CUDA launch failed",
    4: "invalid argument", 5: "workspace missing or too small", 6: "no usable sm_100 device",
    7: "no memory for another arena chunk",
}

# name -> (restype, argtypes); mirrors include/w2a16_moe.h one for one
c_i32, c_i64, c_f32, c_sz, c_vp = ctypes.c_int, ctypes.c_int64, ctypes.c_float, ctypes.c_size_t, ctypes.c_void_p
SIGNATURES = {
    "w2a16_version": (ctypes.c_char_p, []),
    "w2a16_status_string": (ctypes.c_char_p, [c_i32]),
    "w2a16_moe_gemv_tab": (c_i32, [c_vp, c_i64, c_vp, c_vp, c_vp, c_i32, c_vp, c_vp, c_vp, c_i64,
                                   c_i32, c_i32, c_i32, c_i64, c_i64, c_i64, c_i32, c_i32, c_i32, c_vp, c_vp]),
    "w2a16_moe_gemv_slots": (c_i32, [c_vp, c_i64, c_vp, c_i32, c_i32, c_vp, c_i64, c_vp, c_i64, c_vp, c_i64,
                                     c_vp, c_vp, c_vp, c_i64, c_i32, c_i32, c_i32, c_i32, c_i32, c_i32, c_vp, c_vp]),
    "w2a16_moe_layer_workspace_bytes": (c_sz, [c_i32, c_i32, c_i32, c_i32]),
    "w2a16_moe_layer_workspace_bytes_batched": (c_sz, [c_i32, c_i32, c_i32, c_i32]),
    "w2a16_moe_decode_layer_tab": (c_i32, [c_vp, c_i32, c_i32, c_i32, c_i32, c_vp, c_vp, c_i32,
                                           c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_i32, c_f32,
                                           c_vp, c_vp, c_sz, c_vp, c_vp]),
    "w2a16_moe_decode_layer_slots": (c_i32, [c_vp, c_i32, c_i32, c_i32, c_i32, c_vp, c_vp, c_vp, c_i32, c_i32,
                                             c_vp, c_i64, c_vp, c_i64, c_vp, c_i64,
                                             c_vp, c_i64, c_vp, c_i64, c_vp, c_i64,
                                             c_i32, c_f32, c_vp, c_vp, c_sz, c_vp, c_vp]),
    "w2a16_moe_decode_layer_slots_ex": (c_i32, [c_vp, c_i32, c_i32, c_i32, c_i32, c_vp, c_vp, c_vp, c_i32, c_i32,
                                                c_vp, c_i64, c_vp, c_i64, c_vp, c_i64,
                                                c_vp, c_i64, c_vp, c_i64, c_vp, c_i64,
                                                c_i32, c_f32, c_vp, c_vp, c_sz, c_i32, c_vp, c_vp]),
    "w2a16_moe_decode_layer_slots_ep": (c_i32, [c_vp, c_i32, c_i32, c_i32, c_i32, c_vp, c_vp, c_vp, c_i32, c_i32,
                                                c_vp, c_i64, c_vp, c_i64, c_vp, c_i64,
                                                c_vp, c_i64, c_vp, c_i64, c_vp, c_i64,
                                                c_i32, c_f32, c_vp, c_vp, c_sz, c_i32, c_i32, c_vp, c_vp, c_vp]),
    "w2a16_int8_gemv_from_peers": (c_i32, [c_vp, c_vp, c_vp, c_i32, c_i32, c_i32, c_i32, c_i32, c_vp, c_i64, c_vp,
                                           c_vp]),
    "w2a16_moe_decode_layer_slots_noalloc": (c_i32, [c_vp, c_i32, c_i32, c_i32, c_i32, c_vp, c_vp, c_vp, c_i32, c_i32,
                                                     c_vp, c_i64, c_vp, c_i64, c_vp, c_i64,
                                                     c_vp, c_i64, c_vp, c_i64, c_vp, c_i64,
                                                     c_i32, c_f32, c_vp, c_vp, c_vp]),
    "w2a16_to_word_ncontig": (c_i32, [c_vp, c_vp, c_i32, c_i32, c_i32, c_vp]),
    "w2a16_gather_rows_tab": (c_i32, [c_vp, c_vp, c_i32, c_vp, c_i64, c_vp]),
    "w2a16_allreduce_peers_bf16": (c_i32, [c_vp, c_vp, c_i32, c_i32, c_vp, c_sz, c_i32, c_i32, c_vp, c_vp, ctypes.c_uint,
                                           c_vp]),
    "w2a16_int8_gemv": (c_i32, [c_vp, c_i64, c_vp, c_vp, c_i32, c_i32, c_i32, c_i32, c_i32, c_vp, c_i64,
                                c_vp, c_sz, c_vp]),
    "w2a16_int8_workspace_bytes": (c_sz, [c_i32, c_i32, c_i32]),
    "w2a16_arena_create": (c_i32, [c_i32, c_i64, c_i64, c_i64, c_vp]),
    "w2a16_arena_create_with_driver": (c_i32, [c_vp, c_i32, c_i64, c_i64, c_i64, c_vp]),
    "w2a16_arena_ensure_rows": (c_i32, [c_vp, c_i64, c_vp]),
    "w2a16_arena_shrink_rows": (c_i32, [c_vp, c_i64, c_vp]),
    "w2a16_arena_base": (ctypes.c_uint64, [c_vp]),
    "w2a16_arena_backed_rows": (c_i64, [c_vp]),
    "w2a16_arena_chunk_bytes": (c_i64, [c_vp]),
    "w2a16_arena_destroy": (c_i32, [c_vp]),
}


class Exchange(ctypes.Structure):
    """w2a16_exchange of include/w2a16_moe.h (an expert-parallel exchange channel)."""
    _fields_ = [
        ("peer_bufs", c_vp),
        ("tag_offset", c_sz),
        ("n_max", c_i32),
        ("rank", c_i32),
        ("world", c_i32),
        ("epoch", c_vp),
        ("spin_limit", ctypes.c_uint),
    ]


class VmmDriver(ctypes.Structure):
    """w2a16_vmm_driver of include/w2a16_moe.h (a table of driver calls an arena makes)."""
    _u64p = ctypes.POINTER(ctypes.c_uint64)
    _fields_ = [
        ("ctx", c_vp),
        ("granularity", ctypes.CFUNCTYPE(c_i32, c_vp, c_i32, _u64p)),
        ("reserve", ctypes.CFUNCTYPE(c_i32, c_vp, ctypes.c_uint64, _u64p)),
        ("free_va", ctypes.CFUNCTYPE(c_i32, c_vp, ctypes.c_uint64, ctypes.c_uint64)),
        ("create", ctypes.CFUNCTYPE(c_i32, c_vp, c_i32, ctypes.c_uint64, _u64p)),
        ("release", ctypes.CFUNCTYPE(c_i32, c_vp, ctypes.c_uint64)),
        ("map", ctypes.CFUNCTYPE(c_i32, c_vp, c_i32, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_uint64)),
        ("unmap", ctypes.CFUNCTYPE(c_i32, c_vp, ctypes.c_uint64, ctypes.c_uint64)),
    ]

_lib = None
_lock = threading.Lock()


class W2A16Error(RuntimeError):
    """A C-ABI entry point returned a non-zero status."""

    def __init__(self, fn: str, status: int):
        super().__init__(f"{fn} failed: status {status} ({STATUS.get(status, 'unknown')})")
        self.status = status


def lib():
    """Load the shared library once; raise if it is missing (no fallback exists)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(
                    f"W2A16 CUDA library not found at {LIB_PATH}; build it with the package's build.py "
                    "(there is no CPU fallback)")
            h = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                f = getattr(h, name)
                f.restype = res
                f.argtypes = args
            _lib = h
    return _lib


def call(name: str, *args) -> None:
    st = getattr(lib(), name)(*args)
    if st != 0:
        raise W2A16Error(name, st)


def version() -> str:
    return lib().w2a16_version().decode()
