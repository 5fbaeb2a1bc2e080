"""Approved filesystem roots: no-follow, component-by-component file access.

Reference: internal/approved_fs (traversal.c:70-73 openat with O_NOFOLLOW and
a type check per component; identity / snapshot stamps) and
runtime/approved_fs/api.mbt:67-81.  A deployment names an absolute root; every
relative locator is resolved one component at a time with
``openat(dir_fd, name, O_NOFOLLOW)``, so no symlink, ``..`` or absolute
component can leave the root.  ``read_snapshot`` returns the bytes together
with a (device, inode, size, mtime, ctime) stamp and fails if the file changed
while it was read.

``ApprovedRoot`` uses the C++ core (``lunaflux_b200._host.ApprovedRoot``:
the same traversal, reads with the GIL released, ``read_into`` straight into a
caller's buffer such as pinned host memory) when it is built; ``PyApprovedRoot``
is the reference implementation it is tested against.
"""
from __future__ import annotations

import os
import stat
from dataclasses import dataclass
from typing import Tuple


class ApprovedFsError(OSError):
    pass


@dataclass(frozen=True)
class Stamp:
    dev: int
    ino: int
    size: int
    mtime_ns: int
    ctime_ns: int


def _stamp(st) -> Stamp:
    return Stamp(st.st_dev, st.st_ino, st.st_size, st.st_mtime_ns, st.st_ctime_ns)


class PyApprovedRoot:
    """Reference implementation (pure Python, os.open with dir_fd)."""

    def __init__(self, path: str):
        if not os.path.isabs(path):
            raise ApprovedFsError("approved root must be an absolute path")
        try:
            fd = os.open(path, os.O_RDONLY | os.O_DIRECTORY | os.O_NOFOLLOW | os.O_CLOEXEC)
        except OSError as e:
            raise ApprovedFsError(f"cannot open approved root: {e.strerror}") from None
        self.fd = fd
        self.identity = _stamp(os.fstat(fd))

    def close(self):
        if self.fd >= 0:
            os.close(self.fd)
            self.fd = -1

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    def _open(self, locator: str) -> int:
        parts = locator.split("/")
        if not locator or locator.startswith("/") or any(p in ("", ".", "..") for p in parts):
            raise ApprovedFsError("locator must be a relative path without '.', '..' or empty components")
        dfd = self.fd
        opened = []
        try:
            for p in parts[:-1]:
                nfd = os.open(p, os.O_RDONLY | os.O_DIRECTORY | os.O_NOFOLLOW | os.O_CLOEXEC, dir_fd=dfd)
                opened.append(nfd)
                dfd = nfd
            # O_NONBLOCK: opening a FIFO must not wait for a writer (it is rejected below)
            fd = os.open(parts[-1], os.O_RDONLY | os.O_NOFOLLOW | os.O_CLOEXEC | os.O_NONBLOCK, dir_fd=dfd)
        except OSError as e:
            raise ApprovedFsError(f"cannot open locator: {e.strerror}") from None
        finally:
            for f in opened:
                os.close(f)
        if not stat.S_ISREG(os.fstat(fd).st_mode):
            os.close(fd)
            raise ApprovedFsError("locator is not a regular file")
        os.set_blocking(fd, True)
        return fd

    def read_snapshot(self, locator: str, max_bytes: int = 1 << 34) -> Tuple[bytes, Stamp]:
        fd = self._open(locator)
        try:
            before = _stamp(os.fstat(fd))
            if before.size > max_bytes:
                raise ApprovedFsError("file exceeds the size limit")
            chunks = []
            off = 0
            while off < before.size:
                b = os.pread(fd, min(1 << 24, before.size - off), off)
                if not b:
                    break
                chunks.append(b)
                off += len(b)
            data = b"".join(chunks)
            after = _stamp(os.fstat(fd))
            if after != before or len(data) != before.size:
                raise ApprovedFsError("file changed while it was read")
            return data, before
        finally:
            os.close(fd)


class NativeApprovedRoot:
    """The same interface backed by the C++ core."""

    def __init__(self, path: str):
        from .. import _host
        self._h = _host
        try:
            self._r = _host.ApprovedRoot(path)
        except _host.ApprovedFsError as e:
            raise ApprovedFsError(str(e)) from None
        self.identity = Stamp(*self._r.identity())

    def close(self):
        self._r.close()

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    def read_snapshot(self, locator: str, max_bytes: int = 1 << 34) -> Tuple[bytes, Stamp]:
        try:
            data, st = self._r.read_snapshot(locator, max_bytes)
        except self._h.ApprovedFsError as e:
            raise ApprovedFsError(str(e)) from None
        return data, Stamp(*st)

    def stat(self, locator: str) -> Stamp:
        try:
            return Stamp(*self._r.stat(locator))
        except self._h.ApprovedFsError as e:
            raise ApprovedFsError(str(e)) from None

    def read_into(self, locator: str, buf) -> Stamp:
        """Reads the whole file into the start of a writable buffer (e.g. a
        pinned uint8 tensor's numpy view); fails if it does not fit."""
        try:
            return Stamp(*self._r.read_into(locator, buf))
        except self._h.ApprovedFsError as e:
            raise ApprovedFsError(str(e)) from None


def _select():
    try:
        from .. import _host  # noqa: F401
        return NativeApprovedRoot
    except ImportError:
        return PyApprovedRoot


ApprovedRoot = _select()
