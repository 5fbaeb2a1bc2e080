"""Expert parallelism over token-sharded activations: dispatch all-to-all,
grouped expert GEMMs, combine all-to-all.

With sequence parallelism every rank holds the normed rows of its own T / W
tokens.  Each (token, k) routing pair goes to the rank that holds its expert
(E / W experts per rank), the rank runs its experts on everything it received
(one grouped GEMM per projection over all of its experts), and every result
row returns to the rank that owns the token, which forms the top-k weighted
sum.  Per layer and rank this moves each local token to its k experts and
back, about 4 H bytes x k x (W - 1) / W per token, instead of an all-gather
before the experts and a reduce-scatter after them.

``ExpertAllToAll`` runs the exchange with device kernels that store rows
straight into the peers' symmetric buffers (no host round trip, capturable);
``LibraryExpertAllToAll`` is the same path on
``torch.distributed.all_to_all_single`` (the pair counts cross to the host to
size the exchange), which runs on gloo ranks on the CPU and is the baseline
on NCCL.  The experts themselves
go through the same operator set as the tensor-parallel MoE (routing, the
expert-ordered segment alignment padded to 128 rows, the grouped GEMMs).
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.distributed as dist


class LibraryExpertAllToAll:
    def __init__(self, experts: int, topk: int, world: int, rank: int, group=None):
        if experts % world:
            raise ValueError("experts must divide over the expert-parallel ranks")
        self.E, self.k, self.W, self.rank = experts, topk, world, rank
        self.El = experts // world
        self.group = group
        self.calls = 0

    def _a2a(self, out, inp, out_splits, in_splits):
        self.calls += 1
        dist.all_to_all_single(out, inp, out_splits, in_splits, group=self.group)

    def forward(self, h: torch.Tensor, lw, ops, router_bias: Optional[torch.Tensor] = None) -> torch.Tensor:
        """The MoE layer output [T, H] for this rank's token rows h [T, H]."""
        T, H = h.shape
        k, El, W = self.k, self.El, self.W
        dev = h.device
        ids = torch.empty(T, k, dtype=torch.int32, device=dev)
        w = torch.empty(T, k, dtype=torch.float32, device=dev)
        ops.moe_route(h, lw.router, router_bias, k, ids, w)
        flat = ids.view(-1).long()
        dest = flat // El
        n = T * k
        # pairs in destination order (stable: token order within a destination)
        order = torch.argsort(dest * max(n, 1) + torch.arange(n, device=dev))
        send_counts = torch.bincount(dest, minlength=W).to(torch.int64)
        recv_counts = torch.empty_like(send_counts)
        self._a2a(recv_counts, send_counts, None, None)
        sc, rc = send_counts.tolist(), recv_counts.tolist()
        nr = sum(rc)
        send_x = h[order // k].contiguous()
        send_le = (flat[order] - dest[order] * El).to(torch.int32).contiguous()
        recv_x = torch.empty(nr, H, dtype=h.dtype, device=dev)
        recv_le = torch.empty(nr, dtype=torch.int32, device=dev)
        self._a2a(recv_x, send_x, rc, sc)
        self._a2a(recv_le, send_le, rc, sc)
        # this rank's experts on everything it received
        rows = max(128, -(-nr // 128) * 128 + El * 128)
        groups = torch.zeros(El + 1, dtype=torch.int32, device=dev)
        perm = torch.full((rows,), -1, dtype=torch.int32, device=dev)
        slot = torch.full((max(nr, 1),), -1, dtype=torch.int32, device=dev)
        y_recv = torch.zeros(nr, H, dtype=h.dtype, device=dev)
        if nr:
            ops.moe_align(recv_le.view(nr, 1), nr, 1, 0, El, groups, perm, slot)
            F2 = lw.experts_gu.shape[1]
            x = torch.zeros(rows, H, dtype=h.dtype, device=dev)
            act = torch.zeros(rows, F2 // 2, dtype=h.dtype, device=dev)
            y = torch.zeros(rows, H, dtype=h.dtype, device=dev)
            ops.moe_gather(recv_x, perm, groups, El, 1, x)
            ops.gemm_grouped(x, lw.experts_gu, act, groups, El, 2)
            ops.gemm_grouped(act, lw.experts_d, y, groups, El, 0)
            y_recv = y[slot[:nr].long()]
        # results back to the token owners, then the top-k weighted sum
        y_back = torch.empty(n, H, dtype=h.dtype, device=dev)
        self._a2a(y_back, y_recv.contiguous(), sc, rc)
        pairs = torch.empty_like(y_back)
        pairs[order] = y_back
        out = (pairs.view(T, k, H).float() * w.view(T, k, 1)).sum(1)
        return out.to(h.dtype)


class ExpertAllToAll:
    """The same exchange on the GPU with no host round trip: the dispatch and
    combine kernels store rows straight into the peers' symmetric buffers
    (csrc/kernels/moe_a2a.cu), so a layer is capturable in a CUDA graph.
    Buffers are sized for ``max_tokens`` local rows per layer."""

    def __init__(self, experts: int, topk: int, world: int, rank: int, hidden: int, ffn: int, max_tokens: int,
                 device, group=None):
        import torch.distributed._symmetric_memory as symm

        from ..ops import _ext
        if experts % world:
            raise ValueError("experts must divide over the expert-parallel ranks")
        self.C = _ext.load()
        self.E, self.k, self.W, self.rank = experts, topk, world, rank
        self.El = experts // world
        self.H = hidden
        self.cap = max_tokens * topk
        g = group or dist.group.WORLD
        name = g.group_name
        self.recv_x = symm.empty(world * self.cap * hidden, dtype=torch.bfloat16, device=device)
        self.recv_meta = symm.empty(world * self.cap * 2, dtype=torch.int32, device=device)
        self.comb_y = symm.empty(self.cap * hidden, dtype=torch.bfloat16, device=device)
        self.flags = symm.empty(2 * world, dtype=torch.int64, device=device)
        for t in (self.recv_meta, self.flags):
            t.zero_()
        handles = [symm.rendezvous(t, name) for t in (self.recv_x, self.recv_meta, self.comb_y, self.flags)]
        torch.cuda.synchronize(device)
        dist.barrier(group=g)
        hx, hm, hy, hf = handles
        self._handles = handles
        self.ptrs = (list(hx.buffer_ptrs), list(hm.buffer_ptrs), list(hf.buffer_ptrs), list(hy.buffer_ptrs),
                     [p + world * 8 for p in hf.buffer_ptrs])
        self.state = torch.zeros(4, dtype=torch.int32, device=device)
        self.counts = torch.zeros(2 * world, dtype=torch.int32, device=device)
        self.rows_max = -(-world * self.cap // 128) * 128 + self.El * 128
        self.x = torch.zeros(self.rows_max, hidden, dtype=torch.bfloat16, device=device)
        self.act = torch.zeros(self.rows_max, ffn, dtype=torch.bfloat16, device=device)
        self.y = torch.zeros(self.rows_max, hidden, dtype=torch.bfloat16, device=device)
        self.groups = torch.zeros(self.El + 1, dtype=torch.int32, device=device)
        self.perm = torch.full((self.rows_max,), -1, dtype=torch.int32, device=device)
        self.back = torch.zeros(self.rows_max, dtype=torch.int64, device=device)
        self.slot = torch.zeros(self.cap, dtype=torch.int32, device=device)
        self.ids = torch.zeros(max_tokens, topk, dtype=torch.int32, device=device)
        self.w = torch.zeros(max_tokens, topk, dtype=torch.float32, device=device)
        self.out = torch.zeros(max_tokens, hidden, dtype=torch.bfloat16, device=device)
        self.calls = 0

    def _args(self):
        rx, rm, rf, cy, cf = self.ptrs
        return (rx, rm, rf, cy, cf, self.state, self.counts, self.rank, self.El, self.k, self.cap, self.H)

    def forward(self, h: torch.Tensor, lw, ops, router_bias: Optional[torch.Tensor] = None) -> torch.Tensor:
        T = h.shape[0]
        ids, w, out = self.ids[:T], self.w[:T], self.out[:T]
        ops.moe_route(h, lw.router, router_bias, self.k, ids, w)
        a = self._args()
        self.C.moe_a2a_dispatch(h, ids, self.slot, *a)
        self.C.moe_a2a_receive(self.groups, self.perm, self.back, self.x, *a)
        ops.gemm_grouped(self.x, lw.experts_gu, self.act, self.groups, self.El, 2)
        ops.gemm_grouped(self.act, lw.experts_d, self.y, self.groups, self.El, 0)
        self.C.moe_a2a_combine(self.y, self.groups, self.perm, self.back, w, out, *a)
        if hasattr(ops, "launches"):
            ops.launches += 6          # plan, dispatch, receive plan, gather, combine send, combine receive
        self.calls += 1
        return out
