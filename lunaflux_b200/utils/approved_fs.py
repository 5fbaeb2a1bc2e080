"""Approved filesystem roots: no-follow, component-by-component file access.

Reference: internal/approved_fs (traversal.c:70-73 openat with O_NOFOLLOW and
a type check per component; identity / snapshot stamps) and
runtime/approved_fs/api.mbt:67-81.  A deployment names an absolute root; every
relative locator is resolved one component at a time with
``openat(dir_fd, name, O_NOFOLLOW)``, so no symlink, ``..`` or absolute
component can leave the root.  ``read_snapshot`` returns the bytes together
with a (device, inode, size, mtime, ctime) stamp and fails if the file changed
while it was read.
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


class ApprovedRoot:
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
            fd = os.open(parts[-1], os.O_RDONLY | os.O_NOFOLLOW | os.O_CLOEXEC, dir_fd=dfd)
        except OSError as e:
            raise ApprovedFsError(f"cannot open locator: {e.strerror}") from None
        finally:
            for f in opened:
                os.close(f)
        if not stat.S_ISREG(os.fstat(fd).st_mode):
            os.close(fd)
            raise ApprovedFsError("locator is not a regular file")
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
