"""Generational physical KV page allocator.

Reference: kv/page_allocator/allocator.mbt:13-302 and
allocation_checkpoint.mbt:7-107.  Same ownership model:

* ``PageId = (index, generation)``; reuse bumps the generation and stale ids
  are rejected; a slot at the terminal generation is retired, never wrapped.
* Two reference classes: *active* (live requests) and *cached* (prefix-cache
  owners).  A page returns to the FIFO free queue only when both are zero.
* ``checkpoint() / rollback_to() / commit_checkpoint()``: one exclusive
  transaction for provisional allocation; rollback restores the exact FIFO
  order, generations and counts.  Reference-count mutation is rejected while
  a checkpoint is open.

Physical page 0 is reserved by the engine as the all-zero page that padded
rows of a captured batch read; the allocator hands out indices
``[first_index, first_index + capacity)``.
"""
from __future__ import annotations

import collections
from dataclasses import dataclass
from typing import Iterable, List, NamedTuple, Optional


class PageAllocatorError(RuntimeError):
    pass


class OutOfPages(PageAllocatorError):
    pass


class PageId(NamedTuple):
    index: int
    generation: int


FREE, ALLOCATED, RETIRED = 0, 1, 2


@dataclass
class _Checkpoint:
    token: int
    popped: List[int]
    prev_gen: List[int]


class NativePageAllocator:
    """The same allocator backed by the C++ core (``lunaflux_b200._host``)."""

    def __init__(self, capacity: int, first_index: int = 1, max_generation: int = (1 << 31) - 1,
                 max_active_refs: int = 1 << 20, max_cached_refs: int = 1 << 20):
        from .. import _host
        self._h = _host
        self._c = self._call(_host.PageAllocator, capacity, first_index, max_generation, max_active_refs,
                             max_cached_refs)
        self.capacity = capacity
        self.first_index = first_index

    def _call(self, fn, *a):
        try:
            return fn(*a)
        except self._h.OutOfPages as e:
            raise OutOfPages(str(e)) from None
        except self._h.PageError as e:
            raise PageAllocatorError(str(e)) from None

    def free_page_count(self) -> int:
        return self._c.free_page_count()

    def allocated_page_count(self) -> int:
        return self._c.allocated_page_count()

    def retired_page_count(self) -> int:
        return self._c.retired_page_count()

    def allocate_one(self) -> PageId:
        return self.allocate_run(1)[0]

    def allocate_run(self, n: int) -> List[PageId]:
        return [PageId(i, g) for i, g in self._call(self._c.allocate_run, n)]

    def retain_active(self, pid: PageId):
        self._call(self._c.retain_active, pid.index, pid.generation)

    def release_active(self, pid: PageId):
        self._call(self._c.release_active, pid.index, pid.generation)

    def release_active_many(self, pids: Iterable[PageId]):
        for p in pids:
            self.release_active(p)

    def check_release_active(self, pids: Iterable[PageId]):
        self._call(self._c.check_release_active, [(p.index, p.generation) for p in pids])

    def retain_cached(self, pid: PageId):
        self._call(self._c.retain_cached, pid.index, pid.generation)

    def release_cached(self, pid: PageId):
        self._call(self._c.release_cached, pid.index, pid.generation)

    def active_reference_count(self, pid: PageId) -> int:
        return self._call(self._c.active_reference_count, pid.index, pid.generation)

    def cached_reference_count(self, pid: PageId) -> int:
        return self._call(self._c.cached_reference_count, pid.index, pid.generation)

    def validate_active(self, pid: PageId) -> bool:
        return self._c.validate_active(pid.index, pid.generation)

    def checkpoint(self) -> int:
        return self._call(self._c.checkpoint)

    def commit_checkpoint(self, token: int):
        self._call(self._c.commit_checkpoint, token)

    def rollback_to(self, token: int):
        self._call(self._c.rollback_to, token)

    @property
    def _free(self):
        return self._c.free_queue()

    def debug_check_invariants(self):
        self._call(self._c.debug_check_invariants)


def native_available() -> bool:
    try:
        from .. import _host  # noqa: F401
        return True
    except ImportError:
        return False


class PyPageAllocator:
    """Reference implementation of the allocator (the spec the C++ core is
    differentially tested against)."""

    def __init__(self, capacity: int, first_index: int = 1, max_generation: int = (1 << 31) - 1,
                 max_active_refs: int = 1 << 20, max_cached_refs: int = 1 << 20):
        if capacity <= 0:
            raise PageAllocatorError("capacity must be positive")
        self.capacity = capacity
        self.first_index = first_index
        self.max_generation = max_generation
        self.max_active_refs = max_active_refs
        self.max_cached_refs = max_cached_refs
        self._gen = [0] * capacity
        self._state = [FREE] * capacity
        self._active = [0] * capacity
        self._cached = [0] * capacity
        self._free = collections.deque(range(capacity))
        self._allocated = 0
        self._retired = 0
        self._ckpt: Optional[_Checkpoint] = None
        self._ckpt_seq = 0

    # -- counters -------------------------------------------------------------
    def free_page_count(self) -> int:
        return len(self._free)

    def allocated_page_count(self) -> int:
        return self._allocated

    def retired_page_count(self) -> int:
        return self._retired

    # -- identity -------------------------------------------------------------
    def _slot(self, pid: PageId) -> int:
        s = pid.index - self.first_index
        if not (0 <= s < self.capacity) or self._gen[s] != pid.generation or self._state[s] != ALLOCATED:
            raise PageAllocatorError("stale or unknown page id")
        return s

    # -- allocation -------------------------------------------------------------
    def allocate_one(self) -> PageId:
        return self.allocate_run(1)[0]

    def allocate_run(self, n: int) -> List[PageId]:
        if n < 0:
            raise PageAllocatorError("negative run")
        if n > len(self._free):
            raise OutOfPages(f"need {n} pages, {len(self._free)} free")
        out = []
        for _ in range(n):
            s = self._free.popleft()
            if self._ckpt is not None:
                self._ckpt.popped.append(s)
                self._ckpt.prev_gen.append(self._gen[s])
            self._state[s] = ALLOCATED
            self._active[s] = 1
            self._allocated += 1
            out.append(PageId(s + self.first_index, self._gen[s]))
        return out

    def _maybe_free(self, s: int):
        if self._active[s] == 0 and self._cached[s] == 0:
            self._allocated -= 1
            if self._gen[s] >= self.max_generation:
                self._state[s] = RETIRED
                self._retired += 1
            else:
                self._gen[s] += 1
                self._state[s] = FREE
                self._free.append(s)

    def _no_ckpt(self):
        if self._ckpt is not None:
            raise PageAllocatorError("reference counts are frozen while a checkpoint is open")

    def retain_active(self, pid: PageId):
        self._no_ckpt()
        s = self._slot(pid)
        if self._active[s] >= self.max_active_refs:
            raise PageAllocatorError("active reference limit")
        self._active[s] += 1

    def release_active(self, pid: PageId):
        self._no_ckpt()
        s = self._slot(pid)
        if self._active[s] <= 0:
            raise PageAllocatorError("no active reference to release")
        self._active[s] -= 1
        self._maybe_free(s)

    def release_active_many(self, pids: Iterable[PageId]):
        for p in pids:
            self.release_active(p)

    def check_release_active(self, pids: Iterable[PageId]):
        """Raises, changing nothing, unless ``release_active`` could run once
        for every entry of ``pids`` (a page listed n times needs n active
        references)."""
        self._no_ckpt()
        need = collections.Counter(self._slot(p) for p in pids)
        for s, n in need.items():
            if self._active[s] < n:
                raise PageAllocatorError("no active reference to release")

    def retain_cached(self, pid: PageId):
        self._no_ckpt()
        s = self._slot(pid)
        if self._cached[s] >= self.max_cached_refs:
            raise PageAllocatorError("cached reference limit")
        self._cached[s] += 1

    def release_cached(self, pid: PageId):
        self._no_ckpt()
        s = self._slot(pid)
        if self._cached[s] <= 0:
            raise PageAllocatorError("no cached reference to release")
        self._cached[s] -= 1
        self._maybe_free(s)

    def active_reference_count(self, pid: PageId) -> int:
        return self._active[self._slot(pid)]

    def cached_reference_count(self, pid: PageId) -> int:
        return self._cached[self._slot(pid)]

    def validate_active(self, pid: PageId) -> bool:
        try:
            return self._active[self._slot(pid)] > 0
        except PageAllocatorError:
            return False

    # -- transactions --------------------------------------------------------------
    def checkpoint(self) -> int:
        if self._ckpt is not None:
            raise PageAllocatorError("a checkpoint is already open")
        self._ckpt_seq += 1
        self._ckpt = _Checkpoint(self._ckpt_seq, [], [])
        return self._ckpt_seq

    def commit_checkpoint(self, token: int):
        if self._ckpt is None or self._ckpt.token != token:
            raise PageAllocatorError("checkpoint token mismatch")
        self._ckpt = None

    def rollback_to(self, token: int):
        c = self._ckpt
        if c is None or c.token != token:
            raise PageAllocatorError("checkpoint token mismatch")
        for s, g in zip(reversed(c.popped), reversed(c.prev_gen)):
            self._state[s] = FREE
            self._active[s] = 0
            self._gen[s] = g
            self._allocated -= 1
            self._free.appendleft(s)
        self._ckpt = None

    # -- diagnostics ---------------------------------------------------------------
    def debug_check_invariants(self):
        free = set(self._free)
        assert len(free) == len(self._free), "duplicate in free queue"
        n_alloc = n_ret = 0
        for s in range(self.capacity):
            st = self._state[s]
            if st == FREE:
                assert s in free and self._active[s] == 0 and self._cached[s] == 0
            elif st == ALLOCATED:
                assert s not in free and (self._active[s] > 0 or self._cached[s] > 0)
                n_alloc += 1
            else:
                assert s not in free
                n_ret += 1
        assert n_alloc == self._allocated and n_ret == self._retired
        assert len(free) + n_alloc + n_ret == self.capacity


def _select():
    import os
    if os.environ.get("LUNAFLUX_HOST_CORE", "native") == "native" and native_available():
        return NativePageAllocator
    return PyPageAllocator


# The serving path uses the C++ core whenever the host extension is built.
PageAllocator = _select()
