"""Process groups and the collective layer of tensor-parallel serving.

One process per GPU; ``torch.distributed`` with the NCCL backend carries the
bootstrap and the library collectives (the measured baseline of the fused
kernels), a gloo group carries host-side control (request admission
broadcast, heartbeats) so a CPU-side failure never blocks a GPU collective.
Every process group is created with a finite timeout.

The reference has no collective layer at all (NCCL is a planned private ABI:
docs/PLAN.md:686, docs/ARCHITECTURE.md:451).
"""
from __future__ import annotations

import datetime
import os
from typing import Optional

import torch
import torch.distributed as dist


def env_rank_world():
    return int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")), int(
        os.environ.get("LOCAL_RANK", "0"))


def init_distributed(backend: str = "nccl", timeout_s: float = 300.0, device_id: Optional[int] = None):
    """Initialises the default process group from the torchrun environment
    (MASTER_ADDR / MASTER_PORT / RANK / WORLD_SIZE) and a gloo control group."""
    rank, world, local = env_rank_world()
    if world == 1:
        return None
    if not dist.is_initialized():
        kw = {}
        if backend == "nccl" and device_id is not None:
            kw["device_id"] = torch.device("cuda", device_id)
        dist.init_process_group(backend=backend, timeout=datetime.timedelta(seconds=timeout_s), **kw)
    ctrl = dist.new_group(backend="gloo", timeout=datetime.timedelta(seconds=timeout_s)) if backend != "gloo" else None
    return ctrl


class TPComm:
    """Library (NCCL) collectives used by the runner between tcgen05 kernels."""

    def __init__(self, group=None, world: Optional[int] = None, rank: Optional[int] = None):
        self.group = group
        self.world = world if world is not None else dist.get_world_size(group)
        self.rank = rank if rank is not None else dist.get_rank(group)
        self._gather_buf = None
        self.calls = 0

    def all_reduce(self, t: torch.Tensor):
        self.calls += 1
        dist.all_reduce(t, group=self.group)

    def all_gather_cols(self, local: torch.Tensor, full: torch.Tensor):
        """full[:, k*Vl:(k+1)*Vl] = local of rank k (vocab-parallel logits)."""
        R, Vl = local.shape
        need = self.world * local.shape[0] * Vl
        if self._gather_buf is None or self._gather_buf.numel() < need or self._gather_buf.device != local.device:
            self._gather_buf = torch.empty(max(need, 1), dtype=local.dtype, device=local.device)
        buf = self._gather_buf[:need].view(self.world * R, Vl)
        self.calls += 1
        dist.all_gather_into_tensor(buf, local.contiguous(), group=self.group)
        full.view(R, self.world, Vl).copy_(buf.view(self.world, R, Vl).transpose(0, 1))

    def all_gather_flat(self, local: torch.Tensor, out: torch.Tensor):
        """out[k * n:(k + 1) * n] = local of rank k."""
        self.calls += 1
        dist.all_gather_into_tensor(out, local, group=self.group)

    def reduce_scatter_rows(self, full: torch.Tensor, local: torch.Tensor):
        """local = rows [rank * n, (rank + 1) * n) of the sum over ranks of
        full [world * n, H] (sequence parallelism: the residual stream is
        sharded by tokens)."""
        self.calls += 1
        dist.reduce_scatter_tensor(local, full, group=self.group)

    def all_gather_rows(self, local: torch.Tensor, full: torch.Tensor):
        """full [world * n, H] = the ranks' local [n, H] blocks in rank order."""
        self.calls += 1
        dist.all_gather_into_tensor(full, local, group=self.group)

    def barrier(self):
        dist.barrier(group=self.group)

    def max_scalar(self, x: float, device) -> float:
        t = torch.tensor([x], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=self.group)
        return float(t.item())
