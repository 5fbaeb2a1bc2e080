"""Fused GEMM + all-reduce over NVLink for the row-parallel projections.

The o_proj and down projections of a tensor-parallel layer produce partial
sums on every rank.  Instead of a GEMM followed by a library all-reduce,
``gemm_allreduce`` runs ONE tcgen05 kernel per rank whose epilogue publishes
each finished output tile in a symmetric buffer, signals the tile to every
rank, waits (bounded) for the same tile of all ranks and reads the sum back
through the NVSwitch fabric with ``multimem.ld_reduce`` (or peer loads when
the fabric offers no multicast), while the MMA warp of the same CTA already
computes its next tile.  Skinny decode shapes use split-K; there the
all-reduce is fused into the persistent split-K finalize kernel.

Buffers: two slots (ping-pong) of [max_rows, hidden] bf16 plus per-piece
int32 arrival counters, allocated with ``torch.distributed._symmetric_memory``
so that every rank has the peer and multicast addresses.  Two slots suffice:
a rank can only re-use a slot after passing the next operation's wait, which
needs every peer to have finished reading the previous contents.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from ..ops import _ext
from .comm import TPComm

COUNTER_CAPACITY = 1 << 16   # pieces (tiles or row chunks) per slot


class FusedTPComm(TPComm):
    """``TPComm`` plus the symmetric buffers of the fused row-parallel GEMMs."""

    fused = True

    def __init__(self, max_rows: int, hidden: int, device, group=None):
        super().__init__(group)
        import torch.distributed._symmetric_memory as symm
        self.C = _ext.load()
        self.max_rows = max_rows
        self.hidden = hidden
        g = group or dist.group.WORLD
        name = g.group_name
        slot_elems = max_rows * hidden
        self.data = symm.empty(2 * slot_elems, dtype=torch.bfloat16, device=device)
        self.cnt = symm.empty(2 * COUNTER_CAPACITY, dtype=torch.int32, device=device)
        self.data.zero_()
        self.cnt.zero_()
        hd = symm.rendezvous(self.data, name)
        hc = symm.rendezvous(self.cnt, name)
        torch.cuda.synchronize(device)
        dist.barrier(group=g)
        self.multicast = bool(getattr(hd, "multicast_ptr", 0)) and bool(getattr(hc, "multicast_ptr", 0))
        dbytes = slot_elems * 2
        cbytes = COUNTER_CAPACITY * 4
        self.slots = []
        for s in range(2):
            self.slots.append(dict(
                local=self.data.data_ptr() + s * dbytes,
                mc=(hd.multicast_ptr + s * dbytes) if self.multicast else 0,
                peers=[p + s * dbytes for p in hd.buffer_ptrs],
                cnt_local=self.cnt.data_ptr() + s * cbytes,
                cnt_mc=(hc.multicast_ptr + s * cbytes) if self.multicast else 0,
                cnt_peers=[p + s * cbytes for p in hc.buffer_ptrs],
            ))
        self._handles = (hd, hc)
        self.op_index = 0

    def begin_forward(self):
        """Every forward has an even number of fused operations, so starting
        each forward on slot 0 keeps the strict slot alternation."""
        self.op_index = 0

    def gemm_allreduce(self, A: torch.Tensor, B: torch.Tensor, out: torch.Tensor, ws=None):
        if A.shape[0] > self.max_rows or B.shape[0] != self.hidden:
            raise ValueError("gemm_allreduce: shape exceeds the symmetric buffer")
        s = self.slots[self.op_index & 1]
        self.op_index += 1
        self.calls += 1
        self.C.gemm_allreduce(A, B, out, ws, s["local"], s["mc"], s["peers"], s["cnt_local"], s["cnt_mc"],
                              s["cnt_peers"], COUNTER_CAPACITY)

    def reduce_partials(self, part: torch.Tensor, out: torch.Tensor):
        """out (bf16) = sum over ranks of this rank's fp32 partial ``part``."""
        if part.shape[0] > self.max_rows or part.shape[1] != self.hidden:
            raise ValueError("reduce_partials: shape exceeds the symmetric buffer")
        s = self.slots[self.op_index & 1]
        self.op_index += 1
        self.calls += 1
        self.C.partials_allreduce(part, out, 1, s["local"], s["mc"], s["peers"], s["cnt_local"], s["cnt_mc"],
                                  s["cnt_peers"], COUNTER_CAPACITY)
