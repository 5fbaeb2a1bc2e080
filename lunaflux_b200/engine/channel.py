"""Framed control channel between the supervisor and its rank processes.

Reference: internal/process (spawn + socketpair + exact framed I/O with
deadlines; process/README.mbt.md:1-20).  One frame per message:

    u32 magic 'LFC1' | u32 payload length | u64 FNV-1a-64(payload) | payload

(little endian).  A partial frame, a bad magic or checksum, or an oversized
length poisons the channel: every later call raises ``ChannelClosed``.  The
C++ core (``lunaflux_b200._host.Channel``) is used when it is built; the
class below is its reference implementation (same wire format, tested side
by side).  ``MessageChannel`` carries the rank-control frames of
``worker_wire`` over either.
"""
from __future__ import annotations

import select
import socket
import struct
import threading
import time
from typing import Optional

from . import worker_wire

MAGIC = 0x3143464C
_HDR = struct.Struct("<IIQ")


class ChannelClosed(ConnectionError):
    pass


class ChannelTimeout(TimeoutError):
    pass


def fnv1a64(data: bytes) -> int:
    h = 1469598103934665603
    for b in data:
        h = ((h ^ b) * 1099511628211) & 0xFFFFFFFFFFFFFFFF
    return h


class PyChannel:
    """Reference implementation of the framed channel."""

    def __init__(self, fd: int, max_frame: int = 64 << 20, frame_timeout_s: float = 10.0):
        self._sock = socket.socket(fileno=socket.dup(fd))
        self._sock.setblocking(False)
        self.max_frame = max_frame
        self.frame_timeout_s = frame_timeout_s
        self._poisoned = False
        self._send_lock = threading.Lock()
        self._recv_lock = threading.Lock()

    def fileno(self) -> int:
        return self._sock.fileno()

    @property
    def closed(self) -> bool:
        return self._sock.fileno() < 0 or self._poisoned

    def close(self):
        self._sock.close()

    def _check(self):
        if self._sock.fileno() < 0:
            raise ChannelClosed("channel is closed")
        if self._poisoned:
            raise ChannelClosed("channel is poisoned by an earlier framing error")

    def _poison(self, why: str, exc=ChannelClosed):
        self._poisoned = True
        raise exc(why)

    def send(self, payload: bytes, timeout_s: float = 10.0):
        with self._send_lock:
            self._check()
            if len(payload) > self.max_frame:
                raise ValueError("frame exceeds the channel's size limit")
            data = memoryview(_HDR.pack(MAGIC, len(payload), fnv1a64(payload)) + payload)
            deadline = time.monotonic() + timeout_s
            while data:
                try:
                    n = self._sock.send(data)
                    data = data[n:]
                except (BlockingIOError, InterruptedError):
                    left = deadline - time.monotonic()
                    if left <= 0 or not select.select([], [self._sock], [], left)[1]:
                        self._poison("send deadline passed mid-frame", ChannelTimeout)
                except OSError:
                    self._poison("peer closed the channel")

    def _read_exact(self, n: int, deadline: float, at_start: bool) -> bytes:
        buf = bytearray()
        while len(buf) < n:
            try:
                b = self._sock.recv(n - len(buf))
            except (BlockingIOError, InterruptedError):
                left = deadline - time.monotonic()
                if left <= 0 or not select.select([self._sock], [], [], left)[0]:
                    self._poison("frame did not complete before its deadline", ChannelTimeout)
                continue
            except OSError:
                self._poison("recv failed")
            if not b:
                self._poison("peer closed the channel" if at_start and not buf else "peer closed the channel mid-frame")
            buf += b
        return bytes(buf)

    def recv(self, timeout_s: float) -> Optional[bytes]:
        with self._recv_lock:
            self._check()
            if not select.select([self._sock], [], [], max(0.0, timeout_s))[0]:
                return None
            deadline = time.monotonic() + self.frame_timeout_s
            magic, length, digest = _HDR.unpack(self._read_exact(_HDR.size, deadline, True))
            if magic != MAGIC:
                self._poison("bad frame magic")
            if length > self.max_frame:
                self._poison("frame length exceeds the limit")
            payload = self._read_exact(length, deadline, False)
            if fnv1a64(payload) != digest:
                self._poison("frame checksum mismatch")
            return payload


def native_channel_available() -> bool:
    try:
        from .. import _host  # noqa: F401
        return True
    except ImportError:
        return False


def open_channel(fd: int, max_frame: int = 64 << 20, frame_timeout_s: float = 10.0, native: Optional[bool] = None):
    """A channel over a connected stream socket descriptor (duplicated)."""
    if native is None:
        native = native_channel_available()
    if native:
        from .. import _host
        return _host.Channel(fd, max_frame, frame_timeout_s)
    return PyChannel(fd, max_frame, frame_timeout_s)


def _closed_errors():
    errs = [ChannelClosed]
    try:
        from .. import _host
        errs.append(_host.ChannelClosed)
    except ImportError:
        pass
    return tuple(errs)


def _timeout_errors():
    errs = [ChannelTimeout]
    try:
        from .. import _host
        errs.append(_host.ChannelTimeout)
    except ImportError:
        pass
    return tuple(errs)


CLOSED_ERRORS = _closed_errors()
TIMEOUT_ERRORS = _timeout_errors()


class MessageChannel:
    """Rank-control messages (``engine/worker_wire.py`` binary frames) over a
    framed channel.  ``recv`` returns None on timeout and raises ``EOFError``
    once the peer is gone, the framing broke or a frame fails validation
    (the supervisor treats all of them as a lost rank)."""

    def __init__(self, sock: socket.socket, send_timeout_s: float = 30.0, native: Optional[bool] = None):
        self._sock = sock  # keeps the descriptor's origin alive until close()
        self._ch = open_channel(sock.fileno(), native=native)
        self.send_timeout_s = send_timeout_s
        self.generation = 0

    def fileno(self) -> int:
        return self._ch.fileno()

    def send(self, msg) -> None:
        try:
            self._ch.send(worker_wire.encode(msg, self.generation), self.send_timeout_s)
        except CLOSED_ERRORS + TIMEOUT_ERRORS as e:
            raise BrokenPipeError(str(e)) from None

    def recv(self, timeout_s: float = 3600.0):
        try:
            data = self._ch.recv(timeout_s)
        except CLOSED_ERRORS + TIMEOUT_ERRORS as e:
            raise EOFError(str(e)) from None
        if data is None:
            return None
        try:
            msg, generation = worker_wire.decode_with_generation(data)
        except worker_wire.WireError as e:
            raise EOFError(str(e)) from None
        if generation != self.generation:
            raise EOFError(f"frame of generation {generation} on a generation {self.generation} channel")
        return msg

    def close(self):
        self._ch.close()
        self._sock.close()
