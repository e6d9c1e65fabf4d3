"""The C-ABI library: it loads, exports every function include/w2a16_moe.h declares, and rejects bad
arguments with status codes before touching the device (no GPU needed)."""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "w2a16_moe.h")


def header_functions():
    txt = open(HEADER).read()
    txt = re.sub(r"/\*.*?\*/", "", txt, flags=re.S)
    return sorted(set(re.findall(r"\b(w2a16_[a-z0-9_]+)\s*\(", txt)))


def test_header_declares_entry_points():
    names = header_functions()
    for n in ("w2a16_moe_gemv_tab", "w2a16_moe_gemv_slots", "w2a16_moe_decode_layer_tab",
              "w2a16_moe_decode_layer_slots", "w2a16_to_word_ncontig", "w2a16_gather_rows_tab",
              "w2a16_int8_gemv"):
        assert n in names


def test_path_constants_mirror_header(pkg):
    txt = open(HEADER).read()
    defs = dict(re.findall(r"#define (W2A16_[A-Z_]+) (\d+)", txt))
    nat = pkg._native
    assert int(defs["W2A16_PATH_AUTO"]) == nat.PATH_AUTO
    assert int(defs["W2A16_PATH_PER_TOKEN"]) == nat.PATH_PER_TOKEN
    assert int(defs["W2A16_PATH_BATCHED"]) == nat.PATH_BATCHED
    assert int(defs["W2A16_BATCHED_AUTO_TOKENS"]) == nat.BATCHED_AUTO_TOKENS


def test_library_exports_every_declared_symbol(pkg):
    lib = pkg._native.lib()
    missing = [n for n in header_functions() if not hasattr(lib, n)]
    assert not missing, missing
    # and the Python binding covers every declared function
    assert set(header_functions()) <= set(pkg._native.SIGNATURES)


def test_version_and_status_strings(pkg):
    assert "sm_100a" in pkg.version()
    lib = pkg._native.lib()
    assert lib.w2a16_status_string(0) == b"ok"
    assert lib.w2a16_status_string(1) == b"unsupported shape"
    assert lib.w2a16_status_string(99) == b"unknown status"


def test_argument_errors_return_status(pkg):
    lib = pkg._native.lib()
    fake = ctypes.c_void_p(0x1000)
    # K not a multiple of 128 -> shape error, before any launch
    st = lib.w2a16_moe_gemv_tab(fake, 64, fake, fake, None, 8, fake, None, fake, 8, 1, 8, 64, 8, 8, 2,
                                1, 0, 1, None, None)
    assert st == 1
    # N not a multiple of 4
    st = lib.w2a16_moe_gemv_tab(fake, 128, fake, fake, None, 8, fake, None, fake, 6, 1, 6, 128, 6, 6, 2,
                                1, 0, 1, None, None)
    assert st == 1
    # missing tables
    st = lib.w2a16_moe_gemv_tab(fake, 128, None, None, None, 8, fake, None, fake, 8, 1, 8, 128, 8, 8, 2,
                                1, 0, 1, None, None)
    assert st == 4
    # R == 0 is a no-op success
    st = lib.w2a16_moe_gemv_tab(fake, 128, fake, fake, None, 8, fake, None, fake, 8, 0, 8, 128, 8, 8, 2,
                                1, 0, 1, None, None)
    assert st == 0
    # decode layer: workspace too small
    st = lib.w2a16_moe_decode_layer_slots(fake, 1, 256, 256, 2, fake, fake, fake, 4, 4, fake, 4096, fake, 256,
                                          None, 0, fake, 4096, fake, 256, None, 0, 0, 1.0, fake, fake, 16,
                                          None, None)
    assert st == 5
    # decode layer: H not a multiple of 128
    st = lib.w2a16_moe_decode_layer_slots(fake, 1, 200, 256, 2, fake, fake, fake, 4, 4, fake, 4096, fake, 256,
                                          None, 0, fake, 4096, fake, 256, None, 0, 0, 1.0, fake, fake, 1 << 20,
                                          None, None)
    assert st == 1
    # decode layer: an arena without slots
    st = lib.w2a16_moe_decode_layer_slots(fake, 1, 256, 256, 2, fake, fake, fake, 4, 0, fake, 4096, fake, 256,
                                          None, 0, fake, 4096, fake, 256, None, 0, 0, 1.0, fake, fake, 1 << 20,
                                          None, None)
    assert st == 4
    # slot form: misaligned arena base
    st = lib.w2a16_moe_gemv_slots(fake, 128, fake, 4, 4, ctypes.c_void_p(0x1004), 64, fake, 64, None, 0, fake,
                                  None, fake, 8, 1, 8, 128, 1, 0, 1, None, None)
    assert st == 2
    # int8: bad group
    st = lib.w2a16_int8_gemv(fake, 256, fake, fake, 100, 128, 1, 256, 64, fake, 64, fake, 1 << 20, None)
    assert st == 1
    # relayout: K not a multiple of 16
    assert lib.w2a16_to_word_ncontig(fake, fake, 1, 8, 24, None) == 1
    # gather: row bytes not a multiple of 16
    assert lib.w2a16_gather_rows_tab(fake, fake, 2, fake, 24, None) == 2


def test_workspace_sizes(pkg):
    lib = pkg._native.lib()
    assert lib.w2a16_moe_layer_workspace_bytes(1, 4096, 1536, 8) >= 8 * 1536 * 4
    # neither INT8 kernel uses global scratch (column slices reduce inside a CTA, K slices inside a cluster)
    assert 0 < lib.w2a16_int8_workspace_bytes(1, 4096, 4096) <= 4096


def test_batched_workspace_sizes(pkg):
    """The batched layer's workspace query: the per-token size below 16 tokens (the batched path's smallest
    token count), from 16 tokens at least that and room for route tables, h and y rows, no more growth of
    the batched part past one 128-token launch, and never less than the per-token path needs."""
    lib = pkg._native.lib()
    H, I, k = 4096, 1536, 8
    per = lambda M: lib.w2a16_moe_layer_workspace_bytes(M, H, I, k)
    bat = lambda M: lib.w2a16_moe_layer_workspace_bytes_batched(M, H, I, k)
    for M in (1, 8, 15):
        assert bat(M) == per(M), M
    for M in (16, 64):
        rows = M * k
        assert bat(M) >= per(M) and bat(M) >= rows * (I * 2 + H * 4)
    assert bat(16) < bat(64) < bat(128) == bat(256)
    assert bat(1024) == max(per(1024), bat(128))     # the size serves both paths


def _slots_ex(lib, M, path, ws_bytes, H=4096, I=1536, k=8):
    fake = ctypes.c_void_p(0x1000)
    return lib.w2a16_moe_decode_layer_slots_ex(fake, M, H, I, k, fake, fake, fake, 256, 256, fake, 4096, fake, 256,
                                               None, 0, fake, 4096, fake, 256, None, 0, 0, 1.0, fake, fake,
                                               ws_bytes, path, None, None)


def test_explicit_path_errors(pkg):
    """w2a16_moe_decode_layer_slots_ex refuses, before any device work: an unknown path (argument), the
    batched path below 16 tokens (shape) or with a workspace smaller than its size (workspace)."""
    nat = pkg._native
    lib = nat.lib()
    assert _slots_ex(lib, 16, 7, 1 << 30) == 4
    assert _slots_ex(lib, 8, nat.PATH_BATCHED, 1 << 30) == 1
    per16 = lib.w2a16_moe_layer_workspace_bytes(16, 4096, 1536, 8)
    assert _slots_ex(lib, 16, nat.PATH_BATCHED, per16) == 5
    # the per-token path with too small a workspace is refused the same way (no launch)
    assert _slots_ex(lib, 16, nat.PATH_PER_TOKEN, 64) == 5


def test_layer_path_choice(pkg):
    """moe_decode_layer's `batched` argument maps to the C ABI's path choice by token count: the library's
    automatic choice (batched from 64 tokens), the batched path from 16 tokens, or never; the workspace it
    hands over is sized for the path taken."""
    ml = pkg.moe_layer
    nat = pkg._native
    lib = nat.lib()
    H, I, k = 4096, 1536, 8
    per = lambda M: lib.w2a16_moe_layer_workspace_bytes(M, H, I, k)
    bat = lambda M: lib.w2a16_moe_layer_workspace_bytes_batched(M, H, I, k)
    for M in (1, 15, 16, 40, 64, 200):
        assert ml._path(M, 0) == nat.PATH_PER_TOKEN
        assert ml._path(M, -1) == nat.PATH_AUTO
        assert ml._path(M, 1) == (nat.PATH_BATCHED if M >= 16 else nat.PATH_PER_TOKEN)
        assert ml._workspace_bytes(M, H, I, k, 0) == per(M)
        assert ml._workspace_bytes(M, H, I, k, -1) == (bat(M) if M >= 64 else per(M))
        assert ml._workspace_bytes(M, H, I, k, 1) == (bat(M) if M >= 16 else per(M))
    assert ml.BATCHED_MIN_TOKENS == nat.BATCHED_AUTO_TOKENS == 64


def _slots_ep(lib, ex, x_from, y_to, M=1, H=4096, I=1536, k=8, ws_bytes=1 << 30):
    fake = ctypes.c_void_p(0x1000)
    return lib.w2a16_moe_decode_layer_slots_ep(fake, M, H, I, k, fake, fake, fake, 256, 256, fake, 4096, fake, 256,
                                               None, 0, fake, 4096, fake, 256, None, 0, 0, 1.0, fake, fake,
                                               ws_bytes, x_from, y_to, ex, None, None)


def test_exchange_entry_points_refuse_bad_channels(pkg):
    """The expert-parallel entry points refuse, before any device work: an exchange mode without a channel, a
    channel whose n_max cannot hold the layer's M x H values, a misaligned tag offset, a rank outside the world
    (argument); the INT8 projection from peers without a channel (argument)."""
    nat = pkg._native
    lib = nat.lib()
    fake = 0x1000
    assert _slots_ep(lib, None, 1, 0) == 4
    assert _slots_ep(lib, None, 0, 1) == 4
    good = nat.Exchange(fake, 4096, 8192, 0, 2, fake, 0)
    small = nat.Exchange(fake, 4096, 1024, 0, 2, fake, 0)          # n_max < M * H
    skew = nat.Exchange(fake, 4100, 8192, 0, 2, fake, 0)           # tag offset not a multiple of 16
    stray = nat.Exchange(fake, 4096, 8192, 2, 2, fake, 0)          # rank 2 of a world of 2
    for ex in (small, skew, stray):
        assert _slots_ep(lib, ctypes.byref(ex), 1, 1) == 4
    # a well-formed channel passes the argument checks and stops at the workspace check (no launch)
    assert _slots_ep(lib, ctypes.byref(good), 1, 1, ws_bytes=64) == 5
    assert lib.w2a16_int8_gemv_from_peers(None, ctypes.c_void_p(fake), ctypes.c_void_p(fake), 128, 128, 1, 4096, 4096,
                                          ctypes.c_void_p(fake), 4096, None, None) == 4
