"""The native row arena's chunk bookkeeping (csrc/w2a16_arena.cu) against a fake virtual-memory driver: no GPU.
The reference's RowArena (gemv/row_arena.py:34-123) is the behaviour checked: a virtual range reserved once for
max_rows rows, a prefix backed in chunks of the device granularity, growth mapping chunks in order, shrink
unmapping and releasing every chunk entirely beyond the rows kept, OOM leaving the chunks already mapped, close
releasing everything."""
import ctypes

import pytest


class FakeVmm:
    """Records every call; physical chunks run out after `budget` creations."""

    def __init__(self, native, gran=2 << 20, budget=None):
        self.gran, self.budget = gran, budget
        self.reserved = {}                 # base -> bytes
        self.mapped = {}                   # va -> (bytes, handle)
        self.live = set()                  # created, not released handles
        self.next_base, self.next_handle = 0x7F0000000000, 1
        self.calls = []
        D = native.VmmDriver
        F = {n: t for n, t in D._fields_}

        def granularity(ctx, dev, out):
            out[0] = self.gran
            return 0

        def reserve(ctx, nbytes, out):
            base = self.next_base
            self.next_base += (nbytes + (1 << 30)) & ~((1 << 30) - 1)
            self.reserved[base] = nbytes
            out[0] = base
            self.calls.append(("reserve", nbytes))
            return 0

        def free_va(ctx, base, nbytes):
            assert self.reserved.pop(base) == nbytes
            assert not any(base <= va < base + nbytes for va in self.mapped), "freeing a range with mappings"
            self.calls.append(("free", nbytes))
            return 0

        def create(ctx, dev, nbytes, out):
            if self.budget is not None and self.budget <= 0:
                return 2                   # out of memory
            if self.budget is not None:
                self.budget -= 1
            assert nbytes % self.gran == 0
            h = self.next_handle
            self.next_handle += 1
            self.live.add(h)
            out[0] = h
            return 0

        def release(ctx, h):
            assert h in self.live and all(m[1] != h for m in self.mapped.values())
            self.live.remove(h)
            return 0

        def map_(ctx, dev, va, nbytes, h):
            assert h in self.live and va not in self.mapped and va % self.gran == 0
            assert any(b <= va and va + nbytes <= b + n for b, n in self.reserved.items()), "map outside the range"
            self.mapped[va] = (nbytes, h)
            self.calls.append(("map", va))
            return 0

        def unmap(ctx, va, nbytes):
            assert self.mapped.pop(va)[0] == nbytes
            self.calls.append(("unmap", va))
            return 0

        self.fns = [F["granularity"](granularity), F["reserve"](reserve), F["free_va"](free_va), F["create"](create),
                    F["release"](release), F["map"](map_), F["unmap"](unmap)]
        self.table = D(None, *self.fns)


def test_arena_grow_shrink_close(pkg):
    fake = FakeVmm(pkg._native)
    a = pkg.arena.RowArena(300_000, 20, chunk_bytes=1 << 20, name="t", driver=fake.table)
    assert a.chunk == 2 << 20 and a.backed_rows == 0                  # chunk rounded up to the granularity
    assert fake.calls == [("reserve", 6 << 20)]                       # 20 rows -> 6 MB -> three chunks reserved
    assert a.row_addr(3) == a.base + 900_000
    assert a.ensure_rows(5) == 2 << 20 and a.backed_rows == 6         # 2 MiB hold 6 whole rows
    assert a.ensure_rows(6) == 0
    assert a.ensure_rows(7) == 2 << 20 and len(fake.mapped) == 2
    assert sorted(fake.mapped) == [a.base, a.base + (2 << 20)]        # mapped in order, back to back
    assert a.ensure_rows(100) == 2 << 20 and a.backed_rows == 20      # clamped to max_rows
    assert a.shrink_rows(7) == 2 << 20 and a.backed_rows == 13        # the third chunk goes back
    assert a.shrink_rows(7) == 0
    assert a.shrink_rows(0) == 4 << 20 and not fake.mapped and not fake.live
    a.ensure_rows(4)
    a.close()
    assert not fake.reserved and not fake.mapped and not fake.live and fake.calls[-1] == ("free", 6 << 20)


def test_arena_out_of_memory_keeps_mapped_chunks(pkg):
    fake = FakeVmm(pkg._native, budget=2)
    a = pkg.arena.RowArena(1 << 20, 10, chunk_bytes=2 << 20, name="oom", driver=fake.table)
    with pytest.raises(pkg.arena.ArenaOOM):
        a.ensure_rows(10)
    assert a.backed_rows == 4 and len(fake.mapped) == 2
    fake.budget = 10
    assert a.ensure_rows(10) == 6 << 20 and a.backed_rows == 10
    a.close()
    assert not fake.live and not fake.reserved


def test_arena_rejects_bad_arguments(pkg):
    fake = FakeVmm(pkg._native)
    with pytest.raises(pkg.W2A16Error):
        pkg.arena.RowArena(0, 10, driver=fake.table)
    lib = pkg._native.lib()
    h = ctypes.c_void_p()
    assert lib.w2a16_arena_create_with_driver(None, 0, 64, 4, 0, ctypes.byref(h)) == 4
    assert lib.w2a16_arena_ensure_rows(None, 1, None) == 4
