"""Monotonic clocks.  Reference: runtime/monotonic_clock (an injectable clock
so that deadlines and timeouts are testable).  The engine, scheduler and
supervisor take any zero-argument callable returning seconds."""
from __future__ import annotations

import threading
import time


class MonotonicClock:
    def __call__(self) -> float:
        return time.monotonic()


class FakeClock:
    """A clock that moves only when told to (thread-safe)."""

    def __init__(self, start: float = 1000.0):
        self._t = float(start)
        self._lock = threading.Lock()

    def __call__(self) -> float:
        with self._lock:
            return self._t

    def advance(self, seconds: float) -> float:
        if seconds < 0:
            raise ValueError("a monotonic clock does not go back")
        with self._lock:
            self._t += seconds
            return self._t
