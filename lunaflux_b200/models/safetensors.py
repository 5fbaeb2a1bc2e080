"""Safetensors reader and writer (no pickle, no external package).

Reference: model/safetensors_reader/reader.mbt:23-217 (checked little-endian
u64 header length, strict JSON, exact integer conversion, payload
accounting) and model/safetensors/metadata.mbt:47-134 (dtype / rank /
checked sizes, duplicate and overlap rejection).  The same checks are made
here; tensors are returned as zero-copy views of an mmap.
"""
from __future__ import annotations

import json
import mmap
import os
import struct
import warnings
from dataclasses import dataclass
from typing import Dict, Iterable, List, Mapping, Optional, Tuple

import numpy as np
import torch

from ..utils.json_strict import loads_strict

MAX_HEADER_BYTES = 100 * 1024 * 1024

_DTYPES = {
    "F32": (torch.float32, 4),
    "F16": (torch.float16, 2),
    "BF16": (torch.bfloat16, 2),
    "F8_E4M3": (torch.float8_e4m3fn, 1),
    "I32": (torch.int32, 4),
    "I64": (torch.int64, 8),
    "U8": (torch.uint8, 1),
    "I8": (torch.int8, 1),
}
_TORCH_TO_ST = {v[0]: k for k, v in _DTYPES.items()}


class SafetensorsError(ValueError):
    """A rejected file.  ``kind`` names the check that failed (the reader's
    typed errors, model/safetensors_reader/reader.mbt): ``missing_length``,
    ``header_too_large``, ``truncated_header``, ``envelope``, ``encoding``,
    ``json``, ``metadata``, ``tensor_field``, ``integer``, ``dtype``,
    ``rank``, ``name``, ``too_many_tensors``, ``byte_range``, ``outside_payload``,
    ``size_mismatch``, ``size_overflow``, ``overlap``, ``payload_mismatch``;
    ``entry`` is the tensor's index in the header (-1 for file-level checks)."""

    def __init__(self, message: str, kind: str = "invalid", entry: int = -1):
        super().__init__(message)
        self.kind = kind
        self.entry = entry


@dataclass(frozen=True)
class ReaderLimits:
    """Bounds checked before the header is decoded or a tensor is admitted."""
    max_header_bytes: int = MAX_HEADER_BYTES
    max_tensor_count: int = 1 << 16
    max_rank: int = 8
    max_name_length: int = 1024
    max_payload_bytes: int = 1 << 40


_I64_MAX = (1 << 63) - 1


def _exact_int(v, entry: int) -> int:
    """A JSON number that is an exact int64 (``2``, ``2.0`` and ``2e0`` are
    the same value; ``2.5``, ``true`` and values past int64 are not)."""
    if type(v) is float and v.is_integer() and abs(v) <= 2.0 ** 63:
        v = int(v)
    if type(v) is not int or not -_I64_MAX - 1 <= v <= _I64_MAX:
        raise SafetensorsError("not an exact int64", "integer", entry)
    return v


@dataclass(frozen=True)
class TensorMeta:
    name: str
    dtype: str
    shape: Tuple[int, ...]
    begin: int
    end: int

    @property
    def nbytes(self) -> int:
        return self.end - self.begin


def declared_header_bytes(prefix: bytes, limits: ReaderLimits = ReaderLimits()) -> int:
    """The header length that an 8-byte little-endian prefix declares, bounded
    by ``max_header_bytes`` (the prefix must be exactly 8 bytes)."""
    if len(prefix) != 8:
        raise SafetensorsError("the length prefix is 8 bytes", "envelope")
    (hlen,) = struct.unpack("<Q", prefix)
    if hlen > _I64_MAX:
        raise SafetensorsError("declared header length overflows", "header_too_large")
    if hlen > limits.max_header_bytes:
        raise SafetensorsError("declared header length above the limit", "header_too_large")
    return hlen


def parse_header(buf: bytes, file_size: int,
                 limits: ReaderLimits = ReaderLimits()) -> Tuple[int, Dict[str, TensorMeta], Dict[str, str]]:
    """Validates the length prefix, the header envelope and JSON, every
    tensor entry, and that the tensors tile the payload exactly (no overlap,
    no hole, no trailing bytes).  ``buf`` holds at least the prefix and the
    header; ``file_size`` is the whole file's size.  Returns (payload start,
    tensors, metadata)."""
    if len(buf) < 8 or file_size < 8:
        raise SafetensorsError("file shorter than the header length field", "missing_length")
    hlen = declared_header_bytes(bytes(buf[:8]), limits)
    if hlen == 0:
        raise SafetensorsError("empty header", "envelope")
    if 8 + hlen > file_size or 8 + hlen > len(buf):
        raise SafetensorsError("header truncated", "truncated_header")
    payload = file_size - 8 - hlen
    if payload > limits.max_payload_bytes:
        raise SafetensorsError("payload above the limit", "outside_payload")
    raw = bytes(buf[8:8 + hlen])
    # envelope: an object that starts the header; only space padding follows it
    body = raw.rstrip(b" ")
    if not body.startswith(b"{") or not body.endswith(b"}"):
        raise SafetensorsError("header is not one JSON object padded with spaces", "envelope")
    try:
        text = raw.decode("utf-8")
    except UnicodeDecodeError:
        raise SafetensorsError("header is not UTF-8", "encoding") from None
    try:
        obj = loads_strict(text)
    except ValueError as e:
        raise SafetensorsError(f"header is not strict JSON: {e}", "json") from None
    if not isinstance(obj, dict):
        raise SafetensorsError("header must be a JSON object", "envelope")
    n_tensors = len(obj) - ("__metadata__" in obj)
    if n_tensors > limits.max_tensor_count:
        raise SafetensorsError("too many tensors", "too_many_tensors")
    metadata = {}
    tensors: Dict[str, TensorMeta] = {}
    idx = -1
    for name, spec in obj.items():
        if name == "__metadata__":
            if not isinstance(spec, dict) or not all(isinstance(v, str) for v in spec.values()):
                raise SafetensorsError("__metadata__ must map strings to strings", "metadata")
            metadata = dict(spec)
            continue
        idx += 1
        if not name or len(name.encode()) > limits.max_name_length:
            raise SafetensorsError("tensor name empty or too long", "name", idx)
        if not isinstance(spec, dict):
            raise SafetensorsError("tensor entry must be an object", "tensor_field", idx)
        if set(spec) - {"dtype", "shape", "data_offsets"}:
            raise SafetensorsError(f"tensor entry {idx} has unexpected fields", "tensor_field", idx)
        if set(spec) != {"dtype", "shape", "data_offsets"}:
            raise SafetensorsError(f"tensor entry {idx} lacks a field", "tensor_field", idx)
        dt = spec["dtype"]
        if not isinstance(dt, str):
            raise SafetensorsError("dtype must be a string", "tensor_field", idx)
        if dt not in _DTYPES:
            raise SafetensorsError(f"unsupported dtype {dt!r}", "dtype", idx)
        shape = spec["shape"]
        offs = spec["data_offsets"]
        if not isinstance(shape, list):
            raise SafetensorsError("shape must be a list", "tensor_field", idx)
        if not isinstance(offs, list) or len(offs) != 2:
            raise SafetensorsError("data_offsets must be a pair", "tensor_field", idx)
        shape = [_exact_int(d, idx) for d in shape]
        offs = [_exact_int(o, idx) for o in offs]
        if len(shape) > limits.max_rank:
            raise SafetensorsError("tensor rank above the limit", "rank", idx)
        if any(d < 0 for d in shape):
            raise SafetensorsError("shape must be non-negative", "integer", idx)
        if offs[0] < 0 or offs[0] > offs[1]:
            raise SafetensorsError("data_offsets is not a byte range", "byte_range", idx)
        if offs[1] > payload:
            raise SafetensorsError("data_offsets outside the payload", "outside_payload", idx)
        n = _DTYPES[dt][1]
        for d in shape:
            n *= d
            if n > _I64_MAX:
                raise SafetensorsError("tensor byte size overflows", "size_overflow", idx)
        if n != offs[1] - offs[0]:
            raise SafetensorsError(f"tensor {idx} size does not match its shape", "size_mismatch", idx)
        tensors[name] = TensorMeta(name, dt, tuple(shape), offs[0], offs[1])
    # The tensors tile the payload: sorted by begin, each starts where the
    # previous ended, and the last ends at the payload's end.
    spans = sorted((m.begin, m.end, m.name) for m in tensors.values() if m.end > m.begin)
    at = 0
    for b, e, nm in spans:
        if b < at:
            raise SafetensorsError(f"tensor {nm!r} overlaps its predecessor", "overlap")
        if b > at:
            raise SafetensorsError("payload has a hole between tensors", "payload_mismatch")
        at = e
    if at != payload:
        raise SafetensorsError("payload has bytes no tensor covers", "payload_mismatch")
    return 8 + hlen, tensors, metadata


class SafetensorsFile:
    """Memory-mapped safetensors file; `tensor(name)` is a zero-copy CPU view."""

    def __init__(self, path: str):
        self.path = path
        self._f = open(path, "rb")
        size = os.fstat(self._f.fileno()).st_size
        self._mm = mmap.mmap(self._f.fileno(), 0, access=mmap.ACCESS_READ) if size else None
        if self._mm is None:
            raise SafetensorsError("empty file")
        self.data_start, self.tensors, self.metadata = parse_header(self._mm[: min(size, MAX_HEADER_BYTES + 8)], size)
        self._stamp = (os.fstat(self._f.fileno()).st_size, os.fstat(self._f.fileno()).st_mtime_ns)

    def keys(self) -> List[str]:
        return list(self.tensors)

    def tensor(self, name: str) -> torch.Tensor:
        m = self.tensors[name]
        dt, _ = _DTYPES[m.dtype]
        start = self.data_start + m.begin
        arr = np.frombuffer(self._mm, dtype=np.uint8, count=m.nbytes, offset=start)
        with warnings.catch_warnings():
            # the view is read-only by construction (the mmap is opened read-only)
            warnings.simplefilter("ignore", UserWarning)
            t = torch.frombuffer(arr, dtype=torch.uint8) if m.nbytes else torch.empty(0, dtype=torch.uint8)
        return t.view(dt).reshape(m.shape)

    def unchanged(self) -> bool:
        st = os.stat(self.path)
        return (st.st_size, st.st_mtime_ns) == self._stamp

    def close(self):
        """Closes the file.  While tensors returned by ``tensor()`` are alive
        the mapping stays (they are views of it) and is unmapped when the
        last of them is freed."""
        if self._mm is not None:
            try:
                self._mm.close()
            except BufferError:
                pass
            self._mm = None
        self._f.close()

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()


def save_file(tensors: Mapping[str, torch.Tensor], path: str, metadata: Optional[Mapping[str, str]] = None):
    """Writes tensors (any device) in name order, 8-byte aligned payloads."""
    header = {}
    if metadata:
        header["__metadata__"] = dict(metadata)
    offset = 0
    blobs = []
    for name in sorted(tensors):
        t = tensors[name].detach().contiguous().cpu()
        if t.dtype not in _TORCH_TO_ST:
            raise SafetensorsError(f"unsupported dtype {t.dtype}")
        b = t.view(torch.uint8).numpy().tobytes() if t.numel() else b""
        header[name] = {"dtype": _TORCH_TO_ST[t.dtype], "shape": list(t.shape),
                        "data_offsets": [offset, offset + len(b)]}
        blobs.append(b)
        offset += len(b)
    h = json.dumps(header, separators=(",", ":")).encode()
    h += b" " * ((8 - len(h) % 8) % 8)
    tmp = path + ".tmp"
    with open(tmp, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)
    os.replace(tmp, path)


def load_file(path: str, device: str = "cpu") -> Dict[str, torch.Tensor]:
    with SafetensorsFile(path) as f:
        return {k: f.tensor(k).clone().to(device) for k in f.keys()}
