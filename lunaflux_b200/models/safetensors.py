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
    pass


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


def parse_header(buf: bytes, file_size: int) -> Tuple[int, Dict[str, TensorMeta], Dict[str, str]]:
    if len(buf) < 8:
        raise SafetensorsError("file shorter than the header length field")
    (hlen,) = struct.unpack("<Q", buf[:8])
    if hlen == 0 or hlen > MAX_HEADER_BYTES or 8 + hlen > file_size:
        raise SafetensorsError("declared header length out of range")
    raw = bytes(buf[8:8 + hlen])
    try:
        obj = loads_strict(raw.decode("utf-8"))
    except (UnicodeDecodeError, ValueError) as e:
        raise SafetensorsError(f"header is not strict JSON: {e}") from None
    if not isinstance(obj, dict):
        raise SafetensorsError("header must be a JSON object")
    payload = file_size - 8 - hlen
    metadata = {}
    tensors: Dict[str, TensorMeta] = {}
    for name, spec in obj.items():
        if name == "__metadata__":
            if not isinstance(spec, dict) or not all(isinstance(v, str) for v in spec.values()):
                raise SafetensorsError("__metadata__ must map strings to strings")
            metadata = dict(spec)
            continue
        if not isinstance(spec, dict) or set(spec) != {"dtype", "shape", "data_offsets"}:
            raise SafetensorsError(f"tensor entry {name!r} has unexpected fields")
        dt = spec["dtype"]
        if dt not in _DTYPES:
            raise SafetensorsError(f"unsupported dtype {dt!r}")
        shape = spec["shape"]
        offs = spec["data_offsets"]
        if (not isinstance(shape, list) or not all(type(d) is int and d >= 0 for d in shape)):
            raise SafetensorsError("shape must be non-negative integers")
        if (not isinstance(offs, list) or len(offs) != 2 or not all(type(o) is int and o >= 0 for o in offs)
                or offs[0] > offs[1] or offs[1] > payload):
            raise SafetensorsError("data_offsets out of range")
        n = 1
        for d in shape:
            n *= d
        if n * _DTYPES[dt][1] != offs[1] - offs[0]:
            raise SafetensorsError(f"tensor {name!r} size does not match its shape")
        tensors[name] = TensorMeta(name, dt, tuple(shape), offs[0], offs[1])
    # Overlap check: sorted by begin, each must start at or after the previous end.
    spans = sorted((m.begin, m.end, m.name) for m in tensors.values() if m.end > m.begin)
    for (b0, e0, n0), (b1, e1, n1) in zip(spans, spans[1:]):
        if b1 < e0:
            raise SafetensorsError(f"tensors {n0!r} and {n1!r} overlap")
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
