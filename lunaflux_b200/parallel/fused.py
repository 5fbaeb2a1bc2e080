"""Fused GEMM + all-reduce over NVLink for the row-parallel projections.

The o_proj and down projections of a tensor-parallel layer produce partial
sums on every rank.  Instead of a GEMM followed by a library all-reduce,
``gemm_allreduce`` runs ONE tcgen05 kernel per rank whose epilogue publishes
each finished output tile in a symmetric buffer and signals the tile's owner
rank (tiles are dealt round-robin over the ranks).  The owner reads the sum of
all ranks' partials through the NVSwitch (``multimem.ld_reduce``) and writes
it into every rank's result region (``multimem.st``); the other ranks' CTAs
go straight on to their next tile, and the MMA warp of every CTA keeps
computing while its epilogue communicates.  Each rank moves about twice the
output size over NVLink whatever the group size: a bandwidth-optimal
all-reduce with no extra launch.  Without multicast support the same steps
use peer loads and stores.

Decode row counts (at most ``ll_rows``) are latency-bound instead: the GEMM
writes fp32 split-K slabs and the finalize kernel runs a low-latency
reduce-scatter + all-gather whose 8-byte words carry the data and the
operation's epoch together (no fences, no flags, no barriers; see
csrc/kernels/allreduce_ll.cu).  Its result lands in a local buffer.

Buffers: two slots (ping-pong), each a partial region and a result region of
[max_rows, hidden] bf16 plus int32 arrival / completion counters, allocated
with ``torch.distributed._symmetric_memory`` so that every rank has the peer
and multicast addresses.  The result of an operation is a view of the result
region, consumed before the operation after next re-uses the slot.  Two slots
suffice: an owner writes a rank's result region of slot s only after that
rank has published a tile of the new operation, so it has finished every
kernel before it, including the consumer of the previous result in slot s;
and an operation ends on every rank only after every owner has read its
partials.
"""
from __future__ import annotations

import os
from typing import Optional

import torch
import torch.distributed as dist

from ..ops import _ext
from .comm import TPComm

COUNTER_CAPACITY = 1 << 16   # pieces (tiles or row chunks) per slot


class FusedTPComm(TPComm):
    """``TPComm`` plus the symmetric buffers of the fused row-parallel GEMMs."""

    fused = True

    def __init__(self, max_rows: int, hidden: int, device, group=None, ll_rows: Optional[int] = None,
                 tile_min_k: Optional[int] = None):
        super().__init__(group)
        import torch.distributed._symmetric_memory as symm
        self.C = _ext.load()
        self.max_rows = max_rows
        self.hidden = hidden
        g = group or dist.group.WORLD
        name = g.group_name
        slot_elems = max_rows * hidden
        # [slot][partial | result][max_rows * hidden]
        self.data = symm.empty(4 * slot_elems, dtype=torch.bfloat16, device=device)
        self.cnt = symm.empty(2 * 2 * COUNTER_CAPACITY, dtype=torch.int32, device=device)
        self.data.zero_()
        self.cnt.zero_()
        hd = symm.rendezvous(self.data, name)
        hc = symm.rendezvous(self.cnt, name)
        torch.cuda.synchronize(device)
        dist.barrier(group=g)
        self.multicast = bool(getattr(hd, "multicast_ptr", 0)) and bool(getattr(hc, "multicast_ptr", 0))
        if os.environ.get("LUNAFLUX_FUSED_MULTICAST", "1") == "0":
            self.multicast = False   # peer loads and stores only
        dbytes = slot_elems * 2
        cbytes = 2 * COUNTER_CAPACITY * 4
        self.slots = []
        for s in range(2):
            part, res = 2 * s * dbytes, (2 * s + 1) * dbytes
            self.slots.append(dict(
                local=self.data.data_ptr() + part,
                mc=(hd.multicast_ptr + part) if self.multicast else 0,
                peers=[p + part for p in hd.buffer_ptrs],
                out_mc=(hd.multicast_ptr + res) if self.multicast else 0,
                out_peers=[p + res for p in hd.buffer_ptrs],
                cnt_local=self.cnt.data_ptr() + s * cbytes,
                cnt_mc=(hc.multicast_ptr + s * cbytes) if self.multicast else 0,
                cnt_peers=[p + s * cbytes for p in hc.buffer_ptrs],
                result=self.data[(2 * s + 1) * slot_elems:(2 * s + 2) * slot_elems],
            ))
        # Low-latency protocol for decode row counts (rows <= ll_rows): inboxes
        # of 8-byte words (bf16 pair + epoch), see csrc/kernels/allreduce_ll.cu.
        if ll_rows is None:
            ll_rows = int(os.environ.get("LUNAFLUX_FUSED_LL_ROWS", str(min(max_rows, 1024))))
        self.ll_rows = ll_rows
        self.ll_pairs = max(self.ll_rows, 1) * hidden // 2
        rs_words = self.ll_pairs + self.world
        self.ll = symm.empty(rs_words + self.ll_pairs, dtype=torch.int64, device=device)
        self.ll.zero_()
        hl = symm.rendezvous(self.ll, name)
        torch.cuda.synchronize(device)
        dist.barrier(group=g)
        self.ll_rs = list(hl.buffer_ptrs)
        self.ll_ag = [p + rs_words * 8 for p in hl.buffer_ptrs]
        self.ll_ag_mc = (hl.multicast_ptr + rs_words * 8) if (self.multicast and getattr(hl, "multicast_ptr", 0)) else 0
        self.ll_state = torch.zeros(2, dtype=torch.int32, device=device)
        self.ll_out = torch.empty(max(self.ll_rows, 1), hidden, dtype=torch.bfloat16, device=device)
        # Prefill rows: the tile path overlaps each tile's reduction with the
        # next tiles' math.  At TP=2 that pays off when a rank's K share is
        # large (Llama-3-8B down, K=7168: 1.17x over GEMM -> NCCL) and not when
        # it is small (o_proj, K=2048: 0.83x), so below tile_min_k the GEMM is
        # followed by the library all-reduce; at TP=8 the library all-reduce
        # is slower and the tile path wins at every K (o_proj K=512: 1.39x,
        # down K=1792: 1.54x).
        if tile_min_k is None:
            tile_min_k = int(os.environ.get("LUNAFLUX_FUSED_TILE_MIN_K", "4096"))
        self.tile_min_k = tile_min_k
        self.lib_out = torch.empty(max_rows, hidden, dtype=torch.bfloat16, device=device)
        self._handles = (hd, hc, hl)
        self.op_index = 0
        self.trace = None   # optional int64 tensor [4 * tiles]: per-tile timeline of the next calls

    def begin_forward(self):
        """Every forward has an even number of fused operations, so starting
        each forward on slot 0 keeps the strict slot alternation (and the
        layer norms' gathered buffers alternate the same way)."""
        self.op_index = 0
        self.ng_index = 0

    def _slot(self):
        s = self.slots[self.op_index & 1]
        self.op_index += 1
        self.calls += 1
        return s

    def _args(self, s):
        return (s["local"], s["mc"], s["peers"], s["out_mc"], s["out_peers"], s["cnt_local"], s["cnt_mc"],
                s["cnt_peers"], self.rank, COUNTER_CAPACITY,
                self.trace.data_ptr() if self.trace is not None else 0)

    def gemm_allreduce(self, A: torch.Tensor, B: torch.Tensor, ws=None) -> torch.Tensor:
        """Returns the [M, hidden] bf16 sum over ranks of A . B^T (a view of the
        slot's result region, valid until the operation after next)."""
        M = A.shape[0]
        if M > self.max_rows or B.shape[0] != self.hidden:
            raise ValueError("gemm_allreduce: shape exceeds the symmetric buffer")
        if M <= self.ll_rows and ws is not None:
            out = self.ll_out[:M]
            self.calls += 1
            self.C.gemm_allreduce_ll(A, B, out, ws, self.ll_rs, self.ll_ag, self.ll_ag_mc, self.ll_state, self.rank, self.ll_pairs)
            return out
        if self.world <= 2 and A.shape[1] < self.tile_min_k:
            # too little math per tile to hide the tile's reduction behind:
            # the GEMM, then the library all-reduce (measured faster here)
            out = self.lib_out[:M]
            self.C.gemm(A, B, out, 0, 0, ws)
            self.all_reduce(out)
            return out
        s = self._slot()
        self.C.gemm_allreduce(A, B, ws, *self._args(s))
        return s["result"][: M * self.hidden].view(M, self.hidden)

    def enable_norm_gather(self, rows_local: int, device):
        """Symmetric buffers of the sequence-parallel RMSNorm with the
        all-gather in its epilogue: three gathered [world * rows_local,
        hidden] buffers (two alternating over the layers, one for the final
        norm) and the per-rank arrival words."""
        import torch.distributed._symmetric_memory as symm
        if getattr(self, "ng_rows", 0) >= rows_local:
            return
        g = self.group or dist.group.WORLD
        full = self.world * rows_local
        self.ng_buf = symm.empty(3 * full * self.hidden, dtype=torch.bfloat16, device=device)
        self.ng_flag = symm.empty(self.world, dtype=torch.int64, device=device)
        self.ng_flag.zero_()
        hb = symm.rendezvous(self.ng_buf, g.group_name)
        hf = symm.rendezvous(self.ng_flag, g.group_name)
        torch.cuda.synchronize(device)
        dist.barrier(group=g)
        nbytes = full * self.hidden * 2
        self.ng_dst = [[p + b * nbytes for p in hb.buffer_ptrs] for b in range(3)]
        self.ng_flags = list(hf.buffer_ptrs)
        self.ng_state = torch.zeros(2, dtype=torch.int32, device=device)
        self.ng_rows = rows_local
        self.ng_index = 0
        self._ng_handles = (hb, hf)

    def norm_gather(self, x: torch.Tensor, residual, w: torch.Tensor, eps: float, final: bool = False) -> torch.Tensor:
        """RMSNorm of this rank's rows x [rows_local, H] (residual added in
        place when given), gathered on every rank: returns the local
        [world * rows_local, H] view, ready for the next projection."""
        rows = x.shape[0]
        if rows > self.ng_rows:
            raise ValueError("norm_gather: more rows than the enabled size")
        b = 2 if final else (self.ng_index & 1)
        if not final:
            self.ng_index += 1
        self.calls += 1
        self.C.norm_gather(x, residual, w, eps, self.ng_dst[b], self.ng_flags, self.ng_state, self.rank)
        # buffer b starts at b * world * ng_rows rows (sized for the largest
        # step); this step's gathered rows are its first world * rows rows
        base = b * self.world * self.ng_rows * self.hidden
        return self.ng_buf[base: base + self.world * rows * self.hidden].view(self.world * rows, self.hidden)

    def gemm_reduce_scatter(self, A: torch.Tensor, B: torch.Tensor, out_local: torch.Tensor) -> bool:
        """out_local [M / world, hidden] = this rank's rows of the sum over
        ranks of A . B^T, by the row-parallel GEMM with the reduce-scatter in
        the kernel (owner-computes tiles dealt by rows).  Returns False, having
        done nothing, when M / world is not a multiple of 128 or the shape
        exceeds the symmetric buffer (the caller then reduces another way)."""
        M = A.shape[0]
        if M % self.world or (M // self.world) % 128 or M > self.max_rows or B.shape[0] != self.hidden:
            return False
        s = self._slot()
        self.C.gemm_reduce_scatter(A, B, out_local, *self._args(s))
        return True

    def reduce_partials(self, part: torch.Tensor) -> torch.Tensor:
        """Returns the bf16 sum over ranks of this rank's fp32 partial ``part``."""
        M, N = part.shape
        if M > self.max_rows or N != self.hidden:
            raise ValueError("reduce_partials: shape exceeds the symmetric buffer")
        if M <= self.ll_rows:
            out = self.ll_out[:M]
            self.calls += 1
            self.C.partials_allreduce_ll(part, 1, out, self.ll_rs, self.ll_ag, self.ll_ag_mc, self.ll_state, self.rank, self.ll_pairs)
            return out
        s = self._slot()
        self.C.partials_allreduce(part, M, N, 1, *self._args(s))
        return s["result"][: M * N].view(M, N)
