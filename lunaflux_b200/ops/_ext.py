"""Loader for the in-tree sm_100a extension (``lunaflux_b200._C``).

On a machine with a CUDA device the extension is mandatory: importing an op
without it raises instead of silently falling back to PyTorch.  On a CPU-only
machine ``available()`` is False and only the CPU reference paths run.
"""
from __future__ import annotations

import importlib

import torch

_ext = None
_err: Exception | None = None


def load():
    """Return the compiled module, raising a clear error if it is missing."""
    global _ext, _err
    if _ext is not None:
        return _ext
    try:
        _ext = importlib.import_module("lunaflux_b200._C")
    except Exception as e:  # pragma: no cover - depends on the build
        _err = e
        raise RuntimeError(
            "lunaflux_b200._C is not built; run `python setup.py build_ext --inplace` "
            f"(import error: {e})") from e
    return _ext


def available() -> bool:
    try:
        load()
        return True
    except RuntimeError:
        return False


def require_cuda_ext():
    """On a CUDA machine the native kernels are the only GPU path."""
    if torch.cuda.is_available():
        return load()
    raise RuntimeError("lunaflux_b200 GPU ops need a CUDA device")
