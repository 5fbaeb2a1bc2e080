"""Static operator registry: every op the engine launches, the compiled
sm_100a entry point that implements it, its dtypes and the capability it
fills.

Reference: kernels/catalog (a closed table of kernel capabilities,
kernels/catalog/README.mbt.md) and kernels/launch_contract (the launch shape
each capability accepts).  The reference loads AOT modules at run time; here
the kernels are compiled into ``lunaflux_b200._C`` for sm_100a, so the table
maps ops to extension entry points and ``validate`` checks at startup that
every one is present.  A missing entry is a startup error: there is no
fallback to another implementation (docs/DEBT_POLICY.md:57-66).
"""
from __future__ import annotations

import dataclasses
from typing import Dict, List, Tuple


@dataclasses.dataclass(frozen=True)
class OpEntry:
    op: str
    symbol: str                 # attribute of lunaflux_b200._C
    dtypes: Tuple[str, ...]
    capability: str             # the reference's capability slot, or what is new here
    source: str                 # implementing source file


OPS: Tuple[OpEntry, ...] = (
    OpEntry("embed", "embed", ("bf16",), "cap 1: token embedding gather", "csrc/kernels/elementwise.cu"),
    OpEntry("rmsnorm", "rmsnorm", ("bf16",), "cap 2: RMSNorm (+ residual add)", "csrc/kernels/elementwise.cu"),
    OpEntry("linear", "gemm", ("bf16",), "cap 3/6: projections and LM head (tcgen05, cluster split-K)",
            "csrc/kernels/gemm_bf16.cu"),
    OpEntry("linear_fp8", "gemm_fp8", ("e4m3",), "new: block-scaled fp8 projections", "csrc/kernels/gemm_fp8.cu"),
    OpEntry("act_quant", "act_quant", ("bf16->e4m3",), "new: per-token 128-channel fp8 quantisation",
            "csrc/kernels/gemm_fp8.cu"),
    OpEntry("rope_kv_write", "rope_kv_write", ("bf16",), "cap 7/8: RoPE and paged KV write",
            "csrc/kernels/elementwise.cu"),
    OpEntry("linear_qkv_rope", "gemm_qkv_rope", ("bf16",),
            "cap 3 + 7/8: QKV projection with RoPE and the paged KV write in the epilogue",
            "csrc/kernels/gemm_bf16_kernel.cuh"),
    OpEntry("swiglu", "swiglu", ("bf16",), "cap 9: SwiGLU (also fused into the gate/up GEMM)",
            "csrc/kernels/elementwise.cu"),
    OpEntry("attn_prefill", "attn_prefill", ("bf16",), "cap 10: paged causal prefill attention",
            "csrc/kernels/attention.cu"),
    OpEntry("attn_decode", "attn_decode", ("bf16",), "cap 10: paged split-KV decode attention",
            "csrc/kernels/attention.cu"),
    OpEntry("argmax", "argmax", ("fp32",), "sampling: greedy", "csrc/kernels/elementwise.cu"),
    OpEntry("argmax_keys", "argmax_keys", ("fp32",), "sampling: vocab-parallel greedy keys",
            "csrc/kernels/elementwise.cu"),
    OpEntry("keys_to_tokens", "keys_to_tokens", ("int64",), "sampling: vocab-parallel greedy merge",
            "csrc/kernels/elementwise.cu"),
    OpEntry("sample", "sample", ("fp32",), "sampling: top-k / top-p / temperature, counter RNG",
            "csrc/kernels/elementwise.cu"),
    OpEntry("topk_keys", "topk_keys", ("fp32",), "sampling: vocab-parallel per-shard candidate keys",
            "csrc/kernels/elementwise.cu"),
    OpEntry("sample_keys", "sample_keys", ("int64",), "sampling: vocab-parallel draw over gathered candidates",
            "csrc/kernels/elementwise.cu"),
    OpEntry("moe_route", "moe_route", ("bf16",), "new: MoE router top-k", "csrc/kernels/moe.cu"),
    OpEntry("moe_align", "moe_align", ("int32",), "new: MoE expert-ordered permutation", "csrc/kernels/moe.cu"),
    OpEntry("moe_gather", "moe_gather", ("bf16",), "new: MoE gather", "csrc/kernels/moe.cu"),
    OpEntry("moe_grouped_linear", "gemm_grouped", ("bf16",), "new: MoE grouped GEMM", "csrc/kernels/gemm_bf16.cu"),
    OpEntry("moe_combine", "moe_combine", ("bf16",), "new: MoE weighted combine", "csrc/kernels/moe.cu"),
    OpEntry("norm_gather", "norm_gather", ("bf16",),
            "cap 2 + all-gather: sequence-parallel RMSNorm storing its rows on every rank", "csrc/kernels/sp_gather.cu"),
    OpEntry("linear_reduce_scatter", "gemm_reduce_scatter", ("bf16",),
            "new: row-parallel GEMM with the reduce-scatter in the kernel", "csrc/kernels/gemm_bf16_kernel.cuh"),
    OpEntry("moe_a2a_dispatch", "moe_a2a_dispatch", ("bf16",),
            "new: expert-parallel dispatch into the expert ranks' memory", "csrc/kernels/moe_a2a.cu"),
    OpEntry("moe_a2a_receive", "moe_a2a_receive", ("bf16",),
            "new: expert-ordered layout of the received rows", "csrc/kernels/moe_a2a.cu"),
    OpEntry("moe_a2a_combine", "moe_a2a_combine", ("bf16",),
            "new: expert outputs back to their tokens, top-k weighted sum", "csrc/kernels/moe_a2a.cu"),
    OpEntry("linear_allreduce", "gemm_allreduce", ("bf16",), "new: GEMM + all-reduce over NVLink (tile path)",
            "csrc/kernels/gemm_bf16.cu"),
    OpEntry("linear_allreduce_ll", "gemm_allreduce_ll", ("bf16",),
            "new: GEMM + low-latency all-reduce over NVLink (decode)", "csrc/kernels/allreduce_ll.cu"),
    OpEntry("partials_allreduce", "partials_allreduce", ("fp32->bf16",), "new: all-reduce of fp32 partials",
            "csrc/kernels/gemm_bf16.cu"),
    OpEntry("partials_allreduce_ll", "partials_allreduce_ll", ("fp32->bf16",),
            "new: low-latency all-reduce of fp32 partials", "csrc/kernels/allreduce_ll.cu"),
    OpEntry("device_error", "read_error", ("int32",), "device error word (bounded waits, bounds checks)",
            "csrc/kernels/runtime.cu"),
    OpEntry("device_report", "device_report", (), "device probe with typed status", "csrc/runtime/device.cpp"),
)


class KernelRegistryError(RuntimeError):
    pass


def table() -> Dict[str, OpEntry]:
    return {e.op: e for e in OPS}


def missing(module) -> List[str]:
    return [e.op for e in OPS if not callable(getattr(module, e.symbol, None))]


def validate(module) -> None:
    """Raises KernelRegistryError naming every op whose entry point is absent."""
    gone = missing(module)
    if gone:
        raise KernelRegistryError("compiled kernels missing for: " + ", ".join(gone) +
                                  " (rebuild with `python setup.py build_ext --inplace`)")


def manifest(module) -> List[str]:
    """One line per op: op, entry point, dtypes, capability, present or not."""
    out = []
    for e in OPS:
        ok = callable(getattr(module, e.symbol, None))
        out.append(f"{e.op:22s} {e.symbol:22s} {','.join(e.dtypes):12s} {'ok ' if ok else 'MISSING'}  {e.capability}")
    return out
