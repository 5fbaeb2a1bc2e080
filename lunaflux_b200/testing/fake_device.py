"""A fake device: the CPU reference ops with host-side fault injection.

Reference: the fake CUDA device of tests/device_worker_alloc (fault modes at
README.md:29-36) and the worker_echo_fail child.  Every GPU-side failure the
engine must survive is produced here without any GPU: a device error word
reported after a given forward (what a bounded in-kernel wait that ran out
reports), an exception from a kernel launch, or a stall long enough to trip a
step timeout.  The engine and supervisor run unchanged on top of it.
"""
from __future__ import annotations

import dataclasses
import time
from typing import Optional

from ..ops.torch_ops import TorchOps

ERR_PEER_TIMEOUT = 2     # the device error codes of csrc/kernels/common.cuh
ERR_HOST_INJECTED = 5


class InjectedLaunchError(RuntimeError):
    pass


@dataclasses.dataclass
class FaultPlan:
    at_forward: int = 0                  # 1-based forward pass that faults (0: never)
    kind: str = "error_word"             # "error_word" | "launch_error" | "stall"
    error_code: int = ERR_PEER_TIMEOUT
    stall_s: float = 0.0


class FakeDeviceOps(TorchOps):
    def __init__(self, plan: Optional[FaultPlan] = None):
        super().__init__()
        self.plan = plan or FaultPlan()
        self.forwards = 0
        self._error = (0, 0)

    def embed(self, *a, **k):
        # one embedding per forward pass: the pass counter
        self.forwards += 1
        p = self.plan
        if p.at_forward and self.forwards == p.at_forward:
            if p.kind == "launch_error":
                raise InjectedLaunchError(f"injected launch failure at forward {self.forwards}")
            if p.kind == "stall":
                time.sleep(p.stall_s)
            if p.kind == "error_word":
                self._error = (p.error_code, self.forwards)
        return super().embed(*a, **k)

    def read_error(self, clear=True):
        e = self._error
        if clear:
            self._error = (0, 0)
        return e

    def inject_error(self, code: int):
        self._error = (int(code), 0)
