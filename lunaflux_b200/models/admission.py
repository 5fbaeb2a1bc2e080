"""Model admission: can this model run on this deployment, and if not, why.

Reference: model/llama_admission (a model spec is admitted against the
device and kernel capabilities before any weight is loaded, with typed
rejection reasons).  Here the checks are those of the sm_100a kernels and
the tensor / expert-parallel plan, plus a memory plan per rank: weights,
the KV arena for the requested context and batch, and the activation
workspace, against the device's memory.
"""
from __future__ import annotations

import dataclasses
import enum
from typing import List, Optional

from .spec import LlamaSpec


class Rejection(enum.Enum):
    HEAD_DIM = "head_dim"                  # attention kernels are built for head_dim 128
    GQA_GROUP = "gqa_group"                # decode attention packs at most 16 query heads per KV head
    TP_HEADS = "tp_heads"                  # query heads not divisible by the TP degree
    TP_KV_HEADS = "tp_kv_heads"            # KV heads neither divisible by TP nor dividing it
    TP_FFN = "tp_ffn"                      # FFN width not divisible by TP
    TP_VOCAB = "tp_vocab"                  # vocabulary not divisible by TP (vocab-parallel LM head)
    TP_WORLD = "tp_world"                  # more than 8 ranks (one NVSwitch domain)
    EP_EXPERTS = "ep_experts"              # experts not divisible by the EP degree
    FP8_BLOCK = "fp8_block"                # block-scaled fp8 needs 128-aligned projection dims
    GEMM_ALIGN = "gemm_align"              # hidden size not a multiple of 256 (GEMM tiles)
    CONTEXT = "context"                    # requested context not in 1..max_position
    BATCH = "batch"                        # batch rows or step tokens not positive
    MEMORY = "memory"                      # weights + KV + workspace exceed the device memory


@dataclasses.dataclass(frozen=True)
class MemoryPlan:
    weight_bytes: int          # per rank
    kv_bytes: int              # per rank, for max_batch sequences of max_context tokens
    workspace_bytes: int       # activations, logits, GEMM workspace (per rank)
    device_bytes: int          # 0: unknown

    @property
    def total(self) -> int:
        return self.weight_bytes + self.kv_bytes + self.workspace_bytes


@dataclasses.dataclass(frozen=True)
class Admission:
    ok: bool
    reasons: List[Rejection]
    details: List[str]
    memory: MemoryPlan


def _elem(spec: LlamaSpec) -> int:
    return 2 if spec.dtype == "bf16" else 4


def memory_plan(spec: LlamaSpec, tp: int, ep: int, max_context: int, max_batch: int, step_tokens: int,
                page: int = 16, device_bytes: int = 0) -> MemoryPlan:
    """Bytes one rank holds.  The weight term follows the runtime layout
    exactly (``models/weights.py`` ``build_runtime``): the embedding table is
    replicated, the LM head holds this rank's vocabulary rows, each FFN shard
    is padded to the 32-row gate/up interleave group, the MoE router is
    fp32, and fp8 projections carry one fp32 scale per 128 x 128 block."""
    e = _elem(spec)
    H, D = spec.hidden, spec.head_dim
    q = spec.heads * D
    kv = spec.kv_heads * D
    tp = max(tp, 1)
    ep = max(ep, 1)

    def pad32(n: int) -> int:
        return -(-n // 32) * 32

    def blocks(o: int, i: int) -> int:
        return -(-o // 128) * -(-i // 128)

    q_l, kv_l = q // tp, max(kv // tp, D)
    attn = [((q_l + 2 * kv_l), H), (H, q_l)]                 # wqkv, wo: (out, in)
    if spec.is_moe:
        f_l = pad32(spec.ffn if ep > 1 else spec.ffn // tp)
        e_l = spec.experts // ep
        mlp_elems = e_l * 3 * H * f_l
        per_layer = (sum(o * i for o, i in attn) + mlp_elems) * e + spec.experts * H * 4
    else:
        f_l = pad32(spec.ffn // tp)
        mats = attn + [(2 * f_l, H), (H, f_l)]
        if spec.fp8_block:
            per_layer = sum(o * i + 4 * blocks(o, i) for o, i in mats)
        else:
            per_layer = sum(o * i for o, i in mats) * e
    per_layer += 2 * H * e                                  # the two RMSNorm weights
    weights = spec.layers * per_layer + spec.vocab * H * e + (spec.vocab // tp) * H * e + H * e
    kv_heads_local = max(1, spec.kv_heads // tp)
    pages = max_batch * -(-max_context // page) + 1        # + the reserved all-zero page
    kv_bytes = spec.layers * 2 * pages * kv_heads_local * page * D * e
    T = step_tokens + max_batch
    ws = T * (4 * H + (q + 2 * kv) // tp + 2 * spec.ffn // tp) * e + max_batch * spec.vocab * 4 // tp
    ws += 512 * 32768 * 4                  # split / all-reduce workspace
    return MemoryPlan(int(weights), int(kv_bytes), int(ws), int(device_bytes))


def admit(spec: LlamaSpec, tp: int = 1, ep: int = 1, max_context: int = 4096, max_batch: int = 256,
          step_tokens: int = 8192, device_bytes: int = 0, reserve_fraction: float = 0.05,
          kernels: bool = True) -> Admission:
    """Checks the model against the kernels (``kernels``: the sm_100a operator
    set; the CPU reference operators take any shape), the parallel plan and
    (when device_bytes > 0) the memory of one device; every failed check is
    listed."""
    reasons: List[Rejection] = []
    details: List[str] = []

    def no(r: Rejection, msg: str):
        reasons.append(r)
        details.append(msg)

    if kernels and spec.head_dim != 128:
        no(Rejection.HEAD_DIM, f"head_dim {spec.head_dim} (kernels support 128)")
    if kernels and spec.heads // spec.kv_heads > 16:
        no(Rejection.GQA_GROUP, f"{spec.heads // spec.kv_heads} query heads per KV head (at most 16)")
    if not 1 <= tp <= 8:
        no(Rejection.TP_WORLD, f"tensor-parallel degree {tp} (1..8 in one NVSwitch domain)")
    else:
        if spec.heads % tp:
            no(Rejection.TP_HEADS, f"{spec.heads} heads over {tp} ranks")
        if not ((spec.kv_heads >= tp and spec.kv_heads % tp == 0) or (spec.kv_heads < tp and tp % spec.kv_heads == 0)):
            no(Rejection.TP_KV_HEADS, f"{spec.kv_heads} KV heads over {tp} ranks")
        if spec.ffn % tp:
            no(Rejection.TP_FFN, f"ffn {spec.ffn} over {tp} ranks")
        if spec.vocab % tp:
            no(Rejection.TP_VOCAB, f"vocab {spec.vocab} over {tp} ranks")
    if not 1 <= ep <= 8:
        no(Rejection.EP_EXPERTS, f"expert-parallel degree {ep} (1..8 in one NVSwitch domain)")
    elif ep > 1 and (not spec.is_moe or spec.experts % ep):
        no(Rejection.EP_EXPERTS, f"{spec.experts} experts over {ep} expert-parallel ranks")
    if kernels and spec.fp8_block and (spec.hidden % 128 or (spec.ffn // max(tp, 1)) % 128 or (spec.heads * spec.head_dim) % 128):
        no(Rejection.FP8_BLOCK, "fp8 projections need hidden, per-rank ffn and heads*head_dim multiples of 128")
    if kernels and spec.hidden % 256:
        no(Rejection.GEMM_ALIGN, f"hidden {spec.hidden} is not a multiple of 256")
    if not 0 < max_context <= spec.max_position:
        no(Rejection.CONTEXT, f"context {max_context} outside 1..max_position {spec.max_position}")
    if max_batch <= 0 or step_tokens <= 0:
        no(Rejection.BATCH, f"max_batch {max_batch} and step_tokens {step_tokens} must be positive")
    if not 0.0 <= reserve_fraction < 1.0:
        raise ValueError("reserve_fraction must be in [0, 1)")
    mem = memory_plan(spec, max(tp, 1), ep, max_context, max_batch, step_tokens, device_bytes=device_bytes)
    if device_bytes > 0 and mem.total > device_bytes * (1.0 - reserve_fraction):
        no(Rejection.MEMORY, f"needs {mem.total / 2**30:.1f} GiB per rank, device has {device_bytes / 2**30:.1f} GiB")
    return Admission(not reasons, reasons, details, mem)


def admit_on_device(spec: LlamaSpec, tp: int = 1, ep: int = 1, device_index: Optional[int] = 0, **kw) -> Admission:
    """admit() with the memory of a probed device (no memory check when none)."""
    from ..runtime.device import DeviceStatus, probe
    r = probe()
    dev_bytes = 0
    if r.status is DeviceStatus.OK and device_index is not None and device_index < len(r.devices):
        dev_bytes = r.devices[device_index].total_bytes
    return admit(spec, tp, ep, device_bytes=dev_bytes, **kw)
