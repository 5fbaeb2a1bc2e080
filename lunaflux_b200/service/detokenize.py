"""Incremental decoded output with stop strings.

Reference: service/incremental_output (owner.mbt:2, patterns.mbt, utf8.mbt):
token pieces are appended as bytes, only complete UTF-8 is released, a stop
string is matched across token and code-point boundaries, any suffix that may
still grow into a stop string is withheld, and the withheld tail is flushed
with the terminal event.  Matching here uses the Knuth-Morris-Pratt failure
function of each stop string, advanced byte by byte, so the scan is linear in
the output and never re-reads released bytes.  Every released delta is
valid UTF-8: bytes that cannot start or continue a scalar (an unknown
token's raw bytes, a stray continuation byte) are published as U+FFFD.
"""
from __future__ import annotations

from typing import List, Optional, Sequence, Tuple


def _kmp_table(p: bytes) -> List[int]:
    f = [0] * len(p)
    k = 0
    for i in range(1, len(p)):
        while k and p[i] != p[k]:
            k = f[k - 1]
        if p[i] == p[k]:
            k += 1
        f[i] = k
    return f


def _utf8_complete_prefix(b: bytes) -> int:
    """Length of the longest prefix of ``b`` that does not end inside a UTF-8 sequence."""
    n = len(b)
    i = n - 1
    back = 0
    while i >= 0 and back < 4 and (b[i] & 0xC0) == 0x80:
        i -= 1
        back += 1
    if i < 0:
        return n
    lead = b[i]
    need = 1 if lead < 0x80 else 2 if (lead & 0xE0) == 0xC0 else 3 if (lead & 0xF0) == 0xE0 else \
        4 if (lead & 0xF8) == 0xF0 else 1
    return n if n - i >= need else i


def _safe(b: bytes) -> bytes:
    """Valid UTF-8 for a released range (it never ends inside a sequence)."""
    try:
        b.decode("utf-8")
        return b
    except UnicodeDecodeError:
        return b.decode("utf-8", errors="replace").encode("utf-8")


class IncrementalOutput:
    def __init__(self, stop_strings: Sequence[bytes] = ()):
        self.stops = [s for s in stop_strings if s]
        self.tables = [_kmp_table(s) for s in self.stops]
        self.state = [0] * len(self.stops)   # matched length per stop string
        self.buf = bytearray()
        self.released = 0
        self.stopped = False

    def push(self, piece: bytes) -> Tuple[bytes, bool]:
        """Appends one token's bytes.  Returns (delta to release, stop hit)."""
        if self.stopped:
            return b"", True
        start = len(self.buf)
        self.buf += piece
        cut = None
        for off in range(start, len(self.buf)):
            c = self.buf[off]
            for j, s in enumerate(self.stops):
                k = self.state[j]
                t = self.tables[j]
                while k and s[k] != c:
                    k = t[k - 1]
                if s[k] == c:
                    k += 1
                if k == len(s):
                    m = off + 1 - len(s)
                    cut = m if cut is None else min(cut, m)
                    k = t[k - 1]
                self.state[j] = k
            if cut is not None:
                break
        if cut is not None:
            self.stopped = True
            delta = _safe(bytes(self.buf[self.released:cut]))
            self.released = cut
            return delta, True
        hold = max(self.state) if self.state else 0
        safe = len(self.buf) - hold
        safe = self.released + _utf8_complete_prefix(bytes(self.buf[self.released:safe]))
        delta = _safe(bytes(self.buf[self.released:safe]))
        self.released = safe
        return delta, False

    def finish(self) -> bytes:
        """Withheld tail for the terminal event (incomplete UTF-8 replaced)."""
        if self.stopped:
            return b""
        tail = bytes(self.buf[self.released:])
        self.released = len(self.buf)
        return tail.decode("utf-8", errors="replace").encode("utf-8")
