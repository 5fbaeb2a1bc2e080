"""Fixed-capacity per-request block tables (logical page -> physical PageId).

Reference: kv/block_table/arena.mbt:12-369 and allocation_checkpoint.mbt:17-166.
Tables live in an arena of generational slots; each table holds at most
``max_pages`` page ids.  Besides the PageIds, the arena keeps a dense
``int32 [capacity, max_pages]`` matrix of physical page indices (generations
stripped, as the reference does before upload:
engine/device_step/README.mbt.md:23-29) that the engine slices directly into
the per-step descriptor without per-row Python loops.

``BlockTableArena`` is the C++ core (``lunaflux_b200._host.BlockTables``,
which owns the matrix; Python sees a numpy view) whenever the host extension
is built; ``PyBlockTableArena`` is the reference implementation it is tested
against.
"""
from __future__ import annotations

from typing import List, NamedTuple, Optional

import numpy as np

from .page_allocator import PageAllocator, PageId


class BlockTableError(RuntimeError):
    pass


class TableId(NamedTuple):
    index: int
    generation: int


class PyBlockTableArena:
    def __init__(self, capacity: int, max_pages: int, tokens_per_page: int = 16):
        self.capacity = capacity
        self.max_pages = max_pages
        self.tokens_per_page = tokens_per_page
        self._gen = [0] * capacity
        self._live = [False] * capacity
        self._pages: List[List[PageId]] = [[] for _ in range(capacity)]
        self._free = list(range(capacity - 1, -1, -1))
        self.matrix = np.zeros((capacity, max_pages), dtype=np.int32)
        self._ckpt = None

    def _slot(self, tid: TableId) -> int:
        if not (0 <= tid.index < self.capacity) or not self._live[tid.index] or self._gen[tid.index] != tid.generation:
            raise BlockTableError("stale or unknown table id")
        return tid.index

    def free_table_count(self) -> int:
        return len(self._free)

    def allocated_table_count(self) -> int:
        return self.capacity - len(self._free)

    def allocate(self) -> TableId:
        if not self._free:
            raise BlockTableError("no free block table")
        s = self._free.pop()
        self._live[s] = True
        self._pages[s] = []
        return TableId(s, self._gen[s])

    def release(self, tid: TableId):
        s = self._slot(tid)
        if self._pages[s]:
            raise BlockTableError("table still owns pages; use reset_and_release")
        self._live[s] = False
        self._gen[s] += 1
        self._free.append(s)

    def page_count(self, tid: TableId) -> int:
        return len(self._pages[self._slot(tid)])

    def pages(self, tid: TableId) -> List[PageId]:
        return list(self._pages[self._slot(tid)])

    def append_pages(self, tid: TableId, pids: List[PageId]):
        s = self._slot(tid)
        n = len(self._pages[s])
        if n + len(pids) > self.max_pages:
            raise BlockTableError("block table full")
        self._pages[s].extend(pids)
        self.matrix[s, n:n + len(pids)] = [p.index for p in pids]

    def page_at(self, tid: TableId, logical: int) -> PageId:
        v = self._pages[self._slot(tid)]
        if not 0 <= logical < len(v):
            raise BlockTableError("logical page out of range")
        return v[logical]

    def resolve_token_position(self, tid: TableId, position: int):
        """(physical page index, offset in page) of a token position."""
        s = self._slot(tid)
        if position < 0:
            raise BlockTableError("negative position")
        lp, off = divmod(position, self.tokens_per_page)
        if lp >= len(self._pages[s]):
            raise BlockTableError("position beyond the table")
        return self._pages[s][lp].index, off

    def truncate(self, tid: TableId, keep: int, allocator: Optional[PageAllocator] = None) -> List[PageId]:
        """Drops the pages from ``keep`` on (releasing their active reference
        when an allocator is given) and returns them.  A release that would
        fail raises before anything changes, in the table or the allocator."""
        s = self._slot(tid)
        if keep < 0:
            raise BlockTableError("negative length")
        dropped = self._pages[s][keep:]
        if not dropped:
            return []
        if allocator is not None:
            allocator.check_release_active(dropped)
        del self._pages[s][keep:]
        self.matrix[s, keep:keep + len(dropped)] = 0
        if allocator is not None:
            for p in dropped:
                allocator.release_active(p)
        return dropped

    def reset_and_release(self, tid: TableId, allocator: PageAllocator):
        self.truncate(tid, 0, allocator)
        self.release(tid)

    # -- transactions: remember lengths, roll back appended suffixes ---------------
    def checkpoint(self):
        if self._ckpt is not None:
            raise BlockTableError("checkpoint already open")
        self._ckpt = {}
        return True

    def note(self, tid: TableId):
        """Record a table's length before a provisional append."""
        if self._ckpt is not None and tid.index not in self._ckpt:
            self._ckpt[tid.index] = len(self._pages[tid.index])

    def commit_checkpoint(self):
        self._ckpt = None

    def rollback(self):
        """Detach every suffix appended since the checkpoint (pages are not released:
        the page allocator's own rollback reclaims them)."""
        for s, n in (self._ckpt or {}).items():
            extra = len(self._pages[s]) - n
            if extra > 0:
                del self._pages[s][n:]
                self.matrix[s, n:n + extra] = 0
        self._ckpt = None


class NativeBlockTableArena:
    """The same arena backed by the C++ core."""

    def __init__(self, capacity: int, max_pages: int, tokens_per_page: int = 16):
        from .. import _host
        self._h = _host
        self._c = _host.BlockTables(capacity, max_pages, tokens_per_page)
        self.capacity = capacity
        self.max_pages = max_pages
        self.tokens_per_page = tokens_per_page
        self.matrix = self._c.matrix()      # view of the core's own matrix

    def _call(self, fn, *a):
        try:
            return fn(*a)
        except self._h.BlockTableError as e:
            raise BlockTableError(str(e)) from None
        except self._h.PageError as e:
            from .page_allocator import PageAllocatorError
            raise PageAllocatorError(str(e)) from None

    def free_table_count(self) -> int:
        return self._c.free_table_count()

    def allocated_table_count(self) -> int:
        return self._c.allocated_table_count()

    def allocate(self) -> TableId:
        return TableId(*self._call(self._c.allocate))

    def release(self, tid: TableId):
        self._call(self._c.release, tid.index, tid.generation)

    def page_count(self, tid: TableId) -> int:
        return self._call(self._c.page_count, tid.index, tid.generation)

    def pages(self, tid: TableId) -> List[PageId]:
        return [PageId(i, g) for i, g in self._call(self._c.pages, tid.index, tid.generation)]

    def append_pages(self, tid: TableId, pids: List[PageId]):
        self._call(self._c.append_pages, tid.index, tid.generation, pids)

    def page_at(self, tid: TableId, logical: int) -> PageId:
        return PageId(*self._call(self._c.page_at, tid.index, tid.generation, logical))

    def resolve_token_position(self, tid: TableId, position: int):
        return self._call(self._c.resolve_token_position, tid.index, tid.generation, position)

    @staticmethod
    def _native_alloc(allocator):
        return getattr(allocator, "_c", None) if allocator is not None and hasattr(allocator, "_h") else None

    def truncate(self, tid: TableId, keep: int, allocator: Optional[PageAllocator] = None) -> List[PageId]:
        na = self._native_alloc(allocator)
        if allocator is not None and na is None and keep >= 0:
            allocator.check_release_active(self.pages(tid)[keep:])   # preflight, as the core does
        dropped = [PageId(i, g) for i, g in self._call(self._c.truncate, tid.index, tid.generation, keep, na)]
        if allocator is not None and na is None:
            for p in dropped:
                allocator.release_active(p)
        return dropped

    def reset_and_release(self, tid: TableId, allocator: PageAllocator):
        na = self._native_alloc(allocator)
        if na is not None:
            self._call(self._c.reset_and_release, tid.index, tid.generation, na)
        else:
            self.truncate(tid, 0, allocator)
            self.release(tid)

    def checkpoint(self):
        self._call(self._c.checkpoint)
        return True

    def note(self, tid: TableId):
        self._c.note(tid.index)

    def commit_checkpoint(self):
        self._c.commit_checkpoint()

    def rollback(self):
        self._c.rollback()

    def debug_check_invariants(self):
        self._call(self._c.debug_check_invariants)


def _select():
    import os
    from .page_allocator import native_available
    if os.environ.get("LUNAFLUX_HOST_CORE", "native") == "native" and native_available():
        return NativeBlockTableArena
    return PyBlockTableArena


BlockTableArena = _select()
