"""Device memory arena: one allocation per pool, sub-allocated for the life
of the engine, with lease accounting.

Reference: internal/cuda/resources.c (allocation create / lease, atomic
LIVE / CLOSING / CLOSED states; close returns BUSY while operations or
children are live: resources.c:402-433, allocation_lease.c:32-73).  Here an
arena is one ``torch.empty`` block; ``take`` hands out aligned views and
counts them as leases until they are garbage-collected; ``close`` refuses
(ArenaBusy) while any lease is live, unless forced, in which case the live
leases are counted as leaks.
"""
from __future__ import annotations

import threading
import weakref
from typing import Sequence

import torch


class ArenaError(RuntimeError):
    pass


class ArenaBusy(ArenaError):
    pass


LIVE, CLOSED = "live", "closed"


class DeviceArena:
    def __init__(self, nbytes: int, device, name: str = "arena", align: int = 256):
        if nbytes <= 0 or align <= 0 or align & (align - 1):
            raise ArenaError("arena size must be positive and alignment a power of two")
        self.name = name
        self.align = align
        self.device = torch.device(device)
        self._buf = torch.empty(nbytes + align, dtype=torch.uint8, device=self.device)
        self.capacity = nbytes + align
        self.used = 0
        self.state = LIVE
        self.live_leases = 0
        self.leaked = 0
        self._lock = threading.Lock()

    def _release(self):
        with self._lock:
            self.live_leases -= 1

    def take(self, shape: Sequence[int], dtype: torch.dtype) -> torch.Tensor:
        """A tensor view of the next aligned bytes (bump allocation)."""
        n = 1
        for s in shape:
            n *= int(s)
        esize = torch.empty((), dtype=dtype).element_size()
        nbytes = n * esize
        with self._lock:
            if self.state != LIVE:
                raise ArenaError(f"arena {self.name} is closed")
            a = max(self.align, esize)
            off = self.used + (-(self._buf.data_ptr() + self.used)) % a   # next aligned address
            if off + nbytes > self.capacity:
                raise ArenaError(f"arena {self.name}: {nbytes} bytes requested, {self.capacity - off} left")
            self.used = off + nbytes
            self.live_leases += 1
        t = self._buf[off:off + nbytes].view(dtype).view(tuple(shape))
        weakref.finalize(t, self._release)
        return t

    def close(self, force: bool = False):
        """Releases the block.  Raises ArenaBusy while leases are live, unless
        forced (the live leases are then recorded as leaked)."""
        with self._lock:
            if self.state == CLOSED:
                return
            if self.live_leases and not force:
                raise ArenaBusy(f"arena {self.name}: {self.live_leases} live leases")
            self.leaked += self.live_leases
            self.state = CLOSED
            self._buf = None
