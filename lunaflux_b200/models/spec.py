"""Validated model specifications and their canonical digests.

Reference: model/spec/llama.mbt:30 (LlamaModelSpec::new) and
model/spec/digest.mbt:100-140 (plan digest = SHA-256 of a canonical encoding
tagged with a schema string; a separate paged variant binds the KV layout).
The canonical encoding here is this framework's own (UTF-8 "key=value" lines
in fixed order); it keeps the reference's structure: schema tag first, then
every shape field, then the dtype and, for the paged variant, the KV layout.
"""
from __future__ import annotations

import dataclasses
import hashlib
import math
from typing import Optional

DENSE_PLAN_SCHEMA = "lunaflux.dense-llama-plan.v2.full-context"
PAGED_PLAN_SCHEMA = "lunaflux.dense-llama-plan.v2.paged"
MOE_PLAN_SCHEMA = "lunaflux.mixtral-plan.v1.paged"


#: bound on every dimension (and on heads * head_dim): sizes stay well inside
#: 32-bit kernel index arithmetic
MAX_DIMENSION = (1 << 31) - 1


class SpecError(ValueError):
    pass


@dataclasses.dataclass(frozen=True)
class LlamaSpec:
    """Dense Llama-family decoder (also the attention part of Mixtral)."""
    hidden: int
    layers: int
    heads: int
    kv_heads: int
    head_dim: int
    ffn: int
    vocab: int
    rope_theta: float = 10000.0
    rms_eps: float = 1e-5
    max_position: int = 4096
    dtype: str = "bf16"          # activations / weights: "bf16" | "fp32"
    tie_embeddings: bool = False
    # Mixture of experts (Mixtral): experts > 0 replaces the MLP by a routed MoE.
    experts: int = 0
    experts_per_token: int = 0
    # Block-scaled fp8 projections: e4m3 weights with one fp32 scale per
    # 128x128 block, e4m3 activations with one scale per token per 128 channels.
    fp8_block: int = 0
    # RoPE frequency scaling: () for none, or ("llama3", factor, low_freq_factor,
    # high_freq_factor, original_max_position) as in Llama 3.1 / 3.2 / 3.3.
    rope_scaling: tuple = ()

    def __post_init__(self):
        pos = [self.hidden, self.layers, self.heads, self.kv_heads, self.head_dim, self.ffn, self.vocab,
               self.max_position]
        if any(type(v) is not int for v in pos + [self.experts, self.experts_per_token, self.fp8_block]):
            raise SpecError("dimensions must be integers")
        if any(v <= 0 or v > MAX_DIMENSION for v in pos):
            raise SpecError(f"all dimensions must be in 1..{MAX_DIMENSION}")
        if self.heads * self.head_dim > MAX_DIMENSION or self.experts < 0 or self.experts > 1024:
            raise SpecError("geometry out of range")
        if self.heads % self.kv_heads != 0:
            raise SpecError("heads must be a multiple of kv_heads (GQA)")
        if self.head_dim % 2 != 0:
            raise SpecError("head_dim must be even for split-half RoPE")
        for v in (self.rope_theta, self.rms_eps):
            if isinstance(v, bool) or not isinstance(v, (int, float)) or not math.isfinite(v):
                raise SpecError("rope_theta and rms_eps must be finite numbers")
        if not (self.rope_theta > 0 and 0 < self.rms_eps < 1):
            raise SpecError("rope_theta must be positive and rms_eps in (0, 1)")
        if self.dtype not in ("bf16", "fp32"):
            raise SpecError("dtype must be bf16 or fp32")
        if self.experts and not (0 < self.experts_per_token <= self.experts):
            raise SpecError("experts_per_token must be in (0, experts]")
        if not self.experts and self.experts_per_token:
            raise SpecError("experts_per_token without experts")
        if self.fp8_block not in (0, 128):
            raise SpecError("fp8 block size must be 128")
        if self.rope_scaling:
            rs = self.rope_scaling
            if len(rs) != 5 or rs[0] != "llama3":
                raise SpecError("rope_scaling must be () or ('llama3', factor, low, high, original_max_position)")
            _, factor, low, high, orig = rs
            if not all(math.isfinite(x) for x in (factor, low, high)) or type(orig) is not int:
                raise SpecError("llama3 rope scaling needs finite factors and an integer original length")
            if not (factor >= 1.0 and 0 < low < high and int(orig) > 0):
                raise SpecError("llama3 rope scaling needs factor >= 1, 0 < low_freq_factor < high_freq_factor")

    # -- derived sizes ------------------------------------------------------
    @property
    def q_size(self) -> int:
        return self.heads * self.head_dim

    @property
    def kv_size(self) -> int:
        return self.kv_heads * self.head_dim

    @property
    def qkv_size(self) -> int:
        return self.q_size + 2 * self.kv_size

    @property
    def is_moe(self) -> bool:
        return self.experts > 0

    @property
    def group(self) -> int:
        return self.heads // self.kv_heads

    def param_count(self) -> int:
        attn = self.hidden * self.qkv_size + self.q_size * self.hidden
        mlp = 3 * self.hidden * self.ffn * (self.experts if self.is_moe else 1)
        router = self.hidden * self.experts if self.is_moe else 0
        per_layer = attn + mlp + router + 2 * self.hidden
        emb = self.vocab * self.hidden * (1 if self.tie_embeddings else 2)
        return self.layers * per_layer + emb + self.hidden

    def kv_bytes_per_token(self, elem_bytes: int = 2) -> int:
        return self.layers * 2 * self.kv_heads * self.head_dim * elem_bytes

    # -- digests --------------------------------------------------------------
    def canonical_encoding(self, schema: Optional[str] = None) -> bytes:
        schema = schema or (MOE_PLAN_SCHEMA if self.is_moe else DENSE_PLAN_SCHEMA)
        # rope_scaling is encoded only when set, so unscaled specs keep their digests
        fields = [("schema", schema)] + [(f.name, getattr(self, f.name)) for f in dataclasses.fields(self)
                                         if f.name != "rope_scaling" or self.rope_scaling]
        return "\n".join(f"{k}={_canon(v)}" for k, v in fields).encode("utf-8")

    def plan_digest(self) -> str:
        return hashlib.sha256(self.canonical_encoding()).hexdigest()

    def paged_plan_digest(self, tokens_per_page: int, layout_version: int) -> str:
        enc = self.canonical_encoding(PAGED_PLAN_SCHEMA if not self.is_moe else MOE_PLAN_SCHEMA)
        enc += f"\ntokens_per_page={tokens_per_page}\nlayout_version={layout_version}".encode()
        return hashlib.sha256(enc).hexdigest()

    def with_layers(self, layers: int) -> "LlamaSpec":
        return dataclasses.replace(self, layers=layers)


def _canon(v) -> str:
    if isinstance(v, tuple):
        return "(" + ",".join(_canon(x) for x in v) + ")"
    if isinstance(v, bool):
        return "true" if v else "false"
    if isinstance(v, float):
        return repr(float(v))
    return str(v)


# ---------------------------------------------------------------------------
# Named shapes (the benchmark configurations).
# ---------------------------------------------------------------------------
def tiny_llama(dtype: str = "fp32") -> LlamaSpec:
    """CPU plumbing model: 2 layers, hidden 64, 4 heads, 2 KV heads, d 16."""
    return LlamaSpec(hidden=64, layers=2, heads=4, kv_heads=2, head_dim=16, ffn=172, vocab=256, rope_theta=10000.0,
                     rms_eps=1e-5, max_position=512, dtype=dtype)


def llama3_8b(dtype: str = "bf16", layers: int = 32) -> LlamaSpec:
    return LlamaSpec(hidden=4096, layers=layers, heads=32, kv_heads=8, head_dim=128, ffn=14336, vocab=128256,
                     rope_theta=500000.0, rms_eps=1e-5, max_position=8192, dtype=dtype)


def llama31_8b(dtype: str = "bf16", layers: int = 32) -> LlamaSpec:
    """Llama 3.1 8B: the Llama 3 8B shape with 128K context through RoPE scaling."""
    return dataclasses.replace(llama3_8b(dtype, layers), max_position=131072,
                               rope_scaling=("llama3", 8.0, 1.0, 4.0, 8192))


def llama3_70b(fp8: bool = True, layers: int = 80) -> LlamaSpec:
    return LlamaSpec(hidden=8192, layers=layers, heads=64, kv_heads=8, head_dim=128, ffn=28672, vocab=128256,
                     rope_theta=500000.0, rms_eps=1e-5, max_position=8192, dtype="bf16",
                     fp8_block=128 if fp8 else 0)


def mixtral_8x7b(layers: int = 32) -> LlamaSpec:
    return LlamaSpec(hidden=4096, layers=layers, heads=32, kv_heads=8, head_dim=128, ffn=14336, vocab=32000,
                     rope_theta=1000000.0, rms_eps=1e-5, max_position=32768, dtype="bf16", experts=8,
                     experts_per_token=2)


PRESETS = {
    "tiny-llama": tiny_llama,
    "llama3-8b": llama3_8b,
    "llama3.1-8b": llama31_8b,
    "llama3-70b-fp8": llama3_70b,
    "mixtral-8x7b": mixtral_8x7b,
}


def rope_inv_freq(head_dim: int, theta: float, scaling: tuple = ()):
    """Per-pair RoPE frequencies (float64 tensor of head_dim / 2): theta^(-2i/D),
    with Llama 3.1's frequency scaling when ``scaling`` is set (Meta's published
    rule: wavelengths shorter than original_max_position / high_freq_factor
    keep their frequency, those longer than original_max_position /
    low_freq_factor are divided by ``factor``, and the band in between is
    interpolated linearly in original_max_position / wavelength)."""
    import torch
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float64) / head_dim))
    if not scaling:
        return inv
    _, factor, low, high, orig = scaling
    wavelen = 2.0 * math.pi / inv
    ratio = float(orig) / wavelen
    smooth = ((ratio - low) / (high - low)).clamp(0.0, 1.0)
    return (1.0 - smooth) * inv / factor + smooth * inv
