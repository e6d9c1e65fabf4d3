"""Native expert arenas: resizable residency whose row addresses never move.

:class:`RowArena` keeps the method names of the reference's ``RowArena`` (gemv/row_arena.py:34-123) --
``ensure_rows``, ``shrink_rows``, ``row_addr``, ``view``, ``backed_rows``, ``close`` -- over the library's C++ arena
(``w2a16_arena_*`` in include/w2a16_moe.h): virtual addresses for ``max_rows`` rows are reserved once and a prefix
of them is backed by physical chunks, mapped on growth and released on shrink.

:class:`ElasticExpertArena` holds one MoE layer's experts in six such arenas (gate_up codes / scales / zero points,
down codes / scales / zero points; one row = one expert's tensor) and addresses them through an int32 slot table
that is rewritten in place, the way ``ExpertElastic.resize_layer`` grows and shrinks a layer
(gemv/expert_elastic.py:198-252): the resident experts are a prefix of a rank order (hottest first), growing copies
the next experts into rows after the resident ones, shrinking drops the tail rows and unmaps their chunks. Its
``arena`` view is an :class:`~.moe_layer.ExpertArena` spanning all reserved rows, so the decode layer -- and a CUDA
graph captured over it -- keeps working across resizes with the same pointers and shapes.
"""
from __future__ import annotations

import ctypes
from typing import Callable, Dict, List, Optional, Sequence

import torch

from . import _native
from .moe_layer import ExpertArena

__all__ = ["ArenaOOM", "RowArena", "ElasticExpertArena"]

_TYPESTR = {torch.uint8: "|u1", torch.int32: "<i4", torch.float16: "<f2", torch.int16: "<i2"}


class ArenaOOM(RuntimeError):
    """The device has no free physical memory for another arena chunk (w2a16_arena_ensure_rows returned
    W2A16_ERR_MEMORY)."""


class _DeviceMemory:
    """A CUDA array interface over a device address range (for zero-copy, non-owning torch views)."""

    def __init__(self, ptr: int, shape, dtype: torch.dtype, owner):
        self.owner = owner                     # keeps the arena alive while views exist
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": _TYPESTR[dtype], "data": (int(ptr), False),
                                         "version": 3, "strides": None}


class RowArena:
    """A device arena of ``max_rows`` rows of ``row_bytes`` whose backed prefix grows and shrinks in chunks
    (``chunk_bytes`` rounded up to the device granularity). ``driver`` (a :class:`_native.VmmDriver`) replaces the
    CUDA driver's virtual-memory calls, for tests without a GPU."""

    def __init__(self, row_bytes: int, max_rows: int, device_id: int = 0, chunk_bytes: int = 4 << 20, name: str = "",
                 driver: Optional[_native.VmmDriver] = None):
        self.row_bytes, self.max_rows, self.device_id, self.name = int(row_bytes), int(max_rows), int(device_id), name
        self._driver = driver
        h = ctypes.c_void_p()
        lib = _native.lib()
        if driver is None:
            st = lib.w2a16_arena_create(self.device_id, self.row_bytes, self.max_rows, int(chunk_bytes),
                                        ctypes.byref(h))
        else:
            st = lib.w2a16_arena_create_with_driver(ctypes.byref(driver), self.device_id, self.row_bytes,
                                                    self.max_rows, int(chunk_bytes), ctypes.byref(h))
        if st == 7:
            raise ArenaOOM(f"{name}: cannot reserve {self.row_bytes * self.max_rows} bytes of addresses")
        if st != 0:
            raise _native.W2A16Error("w2a16_arena_create", st)
        self._h = h
        self.base = int(lib.w2a16_arena_base(h))
        self.chunk = int(lib.w2a16_arena_chunk_bytes(h))

    @property
    def backed_rows(self) -> int:
        return int(_native.lib().w2a16_arena_backed_rows(self._h)) if self._h else 0

    @property
    def backed_bytes(self) -> int:
        return self.chunks_for_rows(self.backed_rows) * self.chunk if self._h else 0

    def row_addr(self, i: int) -> int:
        return self.base + int(i) * self.row_bytes

    def chunks_for_rows(self, n: int) -> int:
        n = min(int(n), self.max_rows)
        return -(-(n * self.row_bytes) // self.chunk) if n > 0 else 0

    def ensure_rows(self, n: int) -> int:
        """Back rows [0, n); returns the bytes newly mapped. ArenaOOM when the device is out of memory (the chunks
        mapped before that stay mapped)."""
        mapped = ctypes.c_int64(0)
        st = _native.lib().w2a16_arena_ensure_rows(self._h, int(n), ctypes.byref(mapped))
        if st == 7:
            raise ArenaOOM(f"{self.name}: no memory for another {self.chunk >> 20} MiB chunk")
        if st != 0:
            raise _native.W2A16Error("w2a16_arena_ensure_rows", st)
        return int(mapped.value)

    def shrink_rows(self, n: int) -> int:
        """Keep rows [0, n) backed and release every chunk entirely beyond; returns the bytes freed. No kernel may
        still read the released rows (synchronise first)."""
        freed = ctypes.c_int64(0)
        _native.call("w2a16_arena_shrink_rows", self._h, int(n), ctypes.byref(freed))
        return int(freed.value)

    def view(self, n_rows: int, tail=(), dtype: torch.dtype = torch.uint8) -> torch.Tensor:
        """Non-owning tensor [n_rows, *tail] over the arena's rows (rows past the backed prefix must not be
        touched). bf16 views are taken as int16 and reinterpreted."""
        want = torch.int16 if dtype == torch.bfloat16 else dtype
        shape = (int(n_rows),) + tuple(int(t) for t in tail)
        elems = 1
        for t in tail:
            elems *= int(t)
        if elems * torch.empty((), dtype=want).element_size() != self.row_bytes:
            raise ValueError(f"{self.name}: a row of {tail} x {dtype} is not {self.row_bytes} bytes")
        t = torch.as_tensor(_DeviceMemory(self.base, shape, want, self), device=torch.device("cuda", self.device_id))
        return t.view(torch.bfloat16) if dtype == torch.bfloat16 else t

    def close(self):
        if getattr(self, "_h", None):
            if self._driver is None:
                torch.cuda.synchronize(self.device_id)
            st = _native.lib().w2a16_arena_destroy(self._h)
            self._h = None
            if st != 0:
                raise _native.W2A16Error("w2a16_arena_destroy", st)

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class ElasticExpertArena:
    """One MoE layer's experts in native arenas: ``E`` experts, at most ``max_slots`` resident, resident set =
    a prefix of a rank order (hottest first) whose i-th expert sits in row i. ``source(e)`` returns expert e's six
    tensors (dict with keys codes13, scales13, zeros13, codes2, scales2, zeros2; host -- preferably pinned -- or
    device) when it must be copied in."""

    KINDS = ("codes13", "scales13", "zeros13", "codes2", "scales2", "zeros2")

    def __init__(self, E: int, H: int, I: int, max_slots: int, device: torch.device, *,  # noqa: E741
                 scale_dtype: torch.dtype = torch.float16, zeros: bool = True, chunk_bytes: int = 4 << 20):
        self.E, self.H, self.I, self.max_slots = E, H, I, max_slots
        self.device = torch.device(device)
        shapes = {"codes13": ((H // 16, 2 * I), torch.int32), "scales13": ((H // 128, 2 * I), scale_dtype),
                  "zeros13": ((H // 128, 2 * I // 4), torch.uint8), "codes2": ((I // 16, H), torch.int32),
                  "scales2": ((I // 128, H), scale_dtype), "zeros2": ((I // 128, H // 4), torch.uint8)}
        if not zeros:
            del shapes["zeros13"], shapes["zeros2"]
        self.shapes = shapes
        self.arenas: Dict[str, RowArena] = {}
        for n, (tail, dt) in shapes.items():
            rb = torch.empty(tail, dtype=dt).numel() * torch.empty((), dtype=dt).element_size()
            self.arenas[n] = RowArena(rb, max_slots, self.device.index or 0, chunk_bytes, name=n)
        self.slots = torch.full((E,), -1, dtype=torch.int32, device=self.device)
        self.order: List[int] = []           # resident experts, row order
        views = {n: self.arenas[n].view(max_slots, tail, dt) for n, (tail, dt) in shapes.items()}
        self.arena = ExpertArena(views["codes13"], views["scales13"], views["codes2"], views["scales2"],
                                 views.get("zeros13"), views.get("zeros2"), self.slots)

    @property
    def S(self) -> int:
        return len(self.order)

    def resize(self, order: Sequence[int], S: int, source: Callable[[int], Dict[str, torch.Tensor]]) -> None:
        """Make order[:S] the resident experts, expert order[i] in row i. Rows whose expert is unchanged keep
        their bytes; growing maps chunks and copies the new rows in (on the current stream); the slot table is
        rewritten in place; shrinking then waits for the device and unmaps the chunks past row S."""
        S = int(S)
        if S > self.max_slots or S > len(order):
            raise ValueError(f"S={S} exceeds max_slots={self.max_slots} or the rank order")
        new = [int(e) for e in order[:S]]
        for a in self.arenas.values():
            a.ensure_rows(S)
        views = {n: getattr(self.arena, n) for n in self.shapes}
        for i, e in enumerate(new):
            if i < len(self.order) and self.order[i] == e:
                continue
            src = source(e)
            for n in self.shapes:
                views[n][i].copy_(src[n], non_blocking=True)
        table = torch.full((self.E,), -1, dtype=torch.int32)
        for i, e in enumerate(new):
            table[e] = i
        self.slots.copy_(table.to(self.device), non_blocking=True)   # in place: captured graphs see it
        shrink = S < len(self.order)
        self.order = new
        if shrink:
            torch.cuda.synchronize(self.device)
            for a in self.arenas.values():
                a.shrink_rows(S)

    def backed_bytes(self) -> int:
        return sum(a.backed_bytes for a in self.arenas.values())

    def close(self):
        for a in self.arenas.values():
            a.close()
