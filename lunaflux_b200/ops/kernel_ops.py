"""The sm_100a operator set: thin wrappers over the ``_C`` extension.

Every call launches on the current CUDA stream and allocates nothing, so the
decode step can be captured into a CUDA graph.  ``launches`` counts the
kernels this process launched through the extension (a graph replay adds the
count recorded while it was captured).
"""
from __future__ import annotations

import os
from typing import Optional

import torch

from . import _ext

EPI_BF16, EPI_F32, EPI_SWIGLU = 0, 1, 2


class KernelOps:
    name = "kernels"

    def __init__(self):
        self.C = _ext.load()
        from .registry import validate
        validate(self.C)   # every op has its compiled entry point, or startup fails
        self.launches = 0
        self.num_sms = torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count
        self._splitk = {}
        # QKV GEMM with RoPE and the paged K / V write in its epilogue (one
        # kernel instead of two); on unless LUNAFLUX_FUSE_QKV_ROPE=0
        self.fuse_qkv_rope = os.environ.get("LUNAFLUX_FUSE_QKV_ROPE") != "0"
        if os.environ.get("LUNAFLUX_CHECK_LAUNCHES") == "1":
            from .launch_contract import install
            install(self)   # every launch admitted against its operand contract first

    def embed(self, ids, table, out, fwd=None):
        """fwd = (slots, first, prev): rows first.. take prev[slot] where slot >= 0."""
        self.launches += 1
        if fwd is None:
            self.C.embed(ids, table, out)
        else:
            self.C.embed(ids, table, out, fwd[0], fwd[1], fwd[2])

    def rmsnorm(self, x, residual, w, out, eps, rows=None):
        """rows: output row i normalises input row rows[i] (no residual write-back)."""
        self.launches += 1
        self.C.rmsnorm(x, residual, w, out, eps, rows)

    def gemm(self, A, B, out, epi: int = EPI_BF16, ws: Optional[torch.Tensor] = None):
        M, N, K = A.shape[0], B.shape[0], A.shape[1]
        if M == 0:
            return
        self.launches += 1   # plain tiles or cluster split-K: one kernel either way
        self.C.gemm(A, B, out, epi, 0, ws)

    def qkv_rope(self, A, B, qkv, positions, slots, cos_sin, kc, vc, Hq, Hkv, page) -> bool:
        """The fused QKV projection; False (nothing launched) when it is off
        or the shape has no whole-head tile plan."""
        if not self.fuse_qkv_rope or A.shape[0] == 0:
            return False
        if self.C.gemm_qkv_rope(A, B, qkv, positions, slots, cos_sin, kc, vc, Hq, Hkv, page):
            self.launches += 1
            return True
        return False

    def rope_kv_write(self, qkv, positions, slots, cos_sin, kc, vc, Hq, Hkv, page):
        self.launches += 1
        self.C.rope_kv_write(qkv, positions, slots, cos_sin, kc, vc, Hq, Hkv, page)

    def attn_prefill(self, q, out, q_start, seq_lens, bt, kc, vc, Hq, Hkv, max_q_len, host=None):
        self.launches += 1
        self.C.attn_prefill(q, out, q_start, seq_lens, bt, kc, vc, Hq, Hkv, max_q_len)

    def decode_splits(self, rows, Hkv, max_seq):
        return self.C.attn_decode_splits(rows, Hkv, max_seq, self.num_sms)

    def attn_decode(self, q, out, tok, seq_lens, bt, kc, vc, Hq, Hkv, splits, part_o, part_lse, host=None):
        self.launches += 2 if splits > 1 else 1
        self.C.attn_decode(q, out, tok, seq_lens, bt, kc, vc, Hq, Hkv, splits, part_o, part_lse)

    def argmax(self, logits, out):
        self.launches += 1
        self.C.argmax(logits, out, None)

    def sample(self, logits, params, out):
        self.launches += 1
        self.C.sample(logits, params, out, None)

    def read_error(self, clear=True):
        return self.C.read_error(clear)

    def argmax_keys(self, logits, id_offset, keys):
        self.launches += 1
        self.C.argmax_keys(logits, id_offset, keys)

    def keys_to_tokens(self, keys, rows, ranks, out):
        self.launches += 1
        self.C.keys_to_tokens(keys, rows, ranks, out)

    def topk_keys(self, logits, id_offset, kc, keys):
        self.launches += 1
        self.C.topk_keys(logits, id_offset, kc, keys)

    def sample_keys(self, keys, rows, ranks, kc, params, out):
        self.launches += 1
        self.C.sample_keys(keys, rows, ranks, kc, params, out)

    # ---------------------------------------------------------------- MoE
    def moe_route(self, h, router, bias, topk, ids, weights):
        self.launches += 1
        self.C.moe_route(h, router, bias, topk, ids, weights)

    def moe_align(self, ids, T, topk, e0, El, groups, perm, slot, align: int = 128):
        self.launches += 1
        self.C.moe_align(ids, T, topk, e0, El, groups, perm, slot, align)

    def moe_gather(self, h, perm, groups, El, topk, out):
        self.launches += 1
        self.C.moe_gather(h, perm, groups, El, topk, out)

    def gemm_grouped(self, A, B, out, groups, num_groups, epi, align: int = 128):
        self.launches += 1
        self.C.gemm_grouped(A, B, out, groups, num_groups, epi, align)

    def moe_combine(self, y, slot, w, T, topk, out):
        self.launches += 1
        self.C.moe_combine(y, slot, w, T, topk, out)

    # ---------------------------------------------------------------- fp8
    def act_quant(self, x, q, s):
        self.launches += 1
        self.C.act_quant(x, q, s)

    def gemm_fp8(self, q, s, w8, sw, out, epi, ws=None):
        """ws: all-zero fp32 split-K workspace (decode shapes split K over the
        idle SMs and add a finalize kernel)."""
        M, N, K = q.shape[0], w8.shape[0], q.shape[1]
        if M == 0:
            return
        splits = 1
        if ws is not None and M * N <= ws.numel():
            splits = self.C.fp8_plan_splits(-(-M // 128) * (N // 128), K // 128, self.num_sms)[0]
        self.launches += 2 if splits > 1 else 1
        self.C.gemm_fp8(q, s, w8, sw, out, epi, ws)
