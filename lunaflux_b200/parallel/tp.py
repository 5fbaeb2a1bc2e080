"""Tensor-parallel sharding plan (Megatron column / row split).

The reference has no parallelism (its TP is the planned "Phase 7",
docs/PLAN.md:676-703: row/column tensor-parallel plan, sharded weight
materialisation directly to each worker, per-rank KV arenas).  This module
is that plan, built B200-first:

* Q heads split evenly over ranks; KV heads split when kv_heads >= tp,
  otherwise each KV head is replicated on tp / kv_heads ranks.
* QKV and gate/up are column-parallel (each rank owns output features);
  o_proj and down are row-parallel (each rank owns input features) and
  produce partial sums that are reduce-scattered (or all-reduced).
* The LM head is vocab-parallel; the sampler works on vocab shards and
  exchanges candidates instead of gathering full logits.
"""
from __future__ import annotations

import dataclasses

from ..models.spec import LlamaSpec


@dataclasses.dataclass(frozen=True)
class TPShard:
    rank: int
    size: int
    spec: LlamaSpec

    def __post_init__(self):
        s = self.spec
        if self.size < 1 or not (0 <= self.rank < self.size):
            raise ValueError("bad tp rank/size")
        if s.heads % self.size:
            raise ValueError(f"heads {s.heads} not divisible by tp {self.size}")
        if s.kv_heads >= self.size and s.kv_heads % self.size:
            raise ValueError("kv_heads not divisible by tp")
        if s.kv_heads < self.size and self.size % s.kv_heads:
            raise ValueError("tp not a multiple of kv_heads")
        if s.ffn % self.size:
            raise ValueError("ffn not divisible by tp")
        if s.vocab % self.size:
            raise ValueError("vocab not divisible by tp")

    @property
    def heads(self) -> int:
        return self.spec.heads // self.size

    @property
    def kv_heads(self) -> int:
        return max(1, self.spec.kv_heads // self.size)

    @property
    def head_range(self):
        return range(self.rank * self.heads, (self.rank + 1) * self.heads)

    @property
    def kv_head_range(self):
        s = self.spec
        if s.kv_heads >= self.size:
            return range(self.rank * self.kv_heads, (self.rank + 1) * self.kv_heads)
        kv = self.rank * s.kv_heads // self.size
        return range(kv, kv + 1)

    @property
    def ffn(self) -> int:
        return self.spec.ffn // self.size

    @property
    def ffn_padded(self) -> int:
        """FFN shard rounded up to the 32-row gate/up interleave group (the
        padding rows are zero, which leaves silu(g) * u and down() exact)."""
        return -(-self.ffn // 32) * 32

    @property
    def ffn_range(self):
        return range(self.rank * self.ffn, (self.rank + 1) * self.ffn)

    @property
    def vocab(self) -> int:
        return self.spec.vocab // self.size

    @property
    def vocab_range(self):
        return range(self.rank * self.vocab, (self.rank + 1) * self.vocab)

    @property
    def qkv_size(self) -> int:
        return (self.heads + 2 * self.kv_heads) * self.spec.head_dim


def shard_rows(w, r: range):
    return w[r.start:r.stop]


def shard_cols(w, r: range):
    return w[:, r.start:r.stop]
