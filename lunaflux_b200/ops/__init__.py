"""Operator sets used by the model runner.

``KernelOps``   the product path: hand-written sm_100a kernels (``_C``).
``TorchOps``    plain PyTorch restatement of the same operator contracts; it
                runs the CPU configuration (no GPU) and is the measured
                PyTorch + cuBLAS baseline on a GPU.  It is never used as a
                silent fallback: a CUDA runner always uses ``KernelOps`` unless
                the baseline is requested explicitly.
"""
from .kernel_ops import KernelOps  # noqa: F401
from .torch_ops import TorchOps  # noqa: F401


def LibraryOps(device):
    """The library baseline operator set (cuBLAS, vLLM flash-attention, torch)."""
    from .library_ops import LibraryOps as _L
    return _L(device)
