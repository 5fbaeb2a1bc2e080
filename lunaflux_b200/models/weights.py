"""Checkpoint tensor names, seeded random initialisation, and conversion of a
checkpoint into the per-rank runtime layout.

Tensor names follow the Hugging Face Llama / Mixtral layout exactly as the
reference binds them (model/llama_weights/bind.mbt:53-107):
``model.embed_tokens.weight``, ``model.layers.{i}.{input_layernorm,
self_attn.{q,k,v,o}_proj, post_attention_layernorm, mlp.{gate,up,down}_proj}
.weight``, ``model.norm.weight``, ``lm_head.weight``; Mixtral adds
``block_sparse_moe.gate.weight`` and ``block_sparse_moe.experts.{e}.w{1,2,3}
.weight``; block-scaled fp8 checkpoints carry ``*.weight_scale_inv``.

Runtime layout (per tensor-parallel rank):
* ``wqkv``  [(Hq + 2 Hkv) * D, H]  Q rows, then K rows, then V rows;
* ``wgu``   [2 F, H] gate and up rows interleaved in groups of 32 so the
  tcgen05 GEMM's SwiGLU epilogue finds gate and up of the same features in
  one tile;
* everything else as in the checkpoint, sliced for the rank.
"""
from __future__ import annotations

import dataclasses
import hashlib
from typing import Callable, Dict, List, Optional, Tuple

import torch

from ..parallel.tp import TPShard
from .spec import LlamaSpec

SWIGLU_GROUP = 32

Source = Callable[[str], torch.Tensor]


def layer_prefix(i: int) -> str:
    return f"model.layers.{i}."


def checkpoint_names(spec: LlamaSpec) -> List[Tuple[str, Tuple[int, ...]]]:
    """Every tensor of a checkpoint of this spec, with its shape."""
    H, D = spec.hidden, spec.head_dim
    out = [("model.embed_tokens.weight", (spec.vocab, H))]
    for i in range(spec.layers):
        p = layer_prefix(i)
        out += [
            (p + "input_layernorm.weight", (H,)),
            (p + "self_attn.q_proj.weight", (spec.heads * D, H)),
            (p + "self_attn.k_proj.weight", (spec.kv_heads * D, H)),
            (p + "self_attn.v_proj.weight", (spec.kv_heads * D, H)),
            (p + "self_attn.o_proj.weight", (H, spec.heads * D)),
            (p + "post_attention_layernorm.weight", (H,)),
        ]
        if spec.is_moe:
            out.append((p + "block_sparse_moe.gate.weight", (spec.experts, H)))
            for e in range(spec.experts):
                q = p + f"block_sparse_moe.experts.{e}."
                out += [(q + "w1.weight", (spec.ffn, H)), (q + "w2.weight", (H, spec.ffn)),
                        (q + "w3.weight", (spec.ffn, H))]
        else:
            out += [(p + "mlp.gate_proj.weight", (spec.ffn, H)), (p + "mlp.up_proj.weight", (spec.ffn, H)),
                    (p + "mlp.down_proj.weight", (H, spec.ffn))]
    out.append(("model.norm.weight", (H,)))
    if not spec.tie_embeddings:
        out.append(("lm_head.weight", (spec.vocab, H)))
    return out


def _name_seed(seed: int, name: str) -> int:
    return int.from_bytes(hashlib.sha256(f"{seed}:{name}".encode()).digest()[:8], "little") & 0x7FFF_FFFF_FFFF


def random_tensor(name: str, shape, seed: int, device="cpu", dtype=torch.float32, std: float = 0.02) -> torch.Tensor:
    """N(0, std) weights (norm weights are ones), reproducible per (seed, name)."""
    if name.endswith("layernorm.weight") or name == "model.norm.weight":
        return torch.ones(shape, device=device, dtype=dtype)
    g = torch.Generator(device=device)
    g.manual_seed(_name_seed(seed, name))
    t = torch.empty(shape, device=device, dtype=torch.float32)
    t.normal_(0.0, std, generator=g)
    return t.to(dtype)


def random_source(spec: LlamaSpec, seed: int = 0, device="cpu", dtype=torch.float32) -> Source:
    shapes = dict(checkpoint_names(spec))

    def get(name: str) -> torch.Tensor:
        return random_tensor(name, shapes[name], seed, device, dtype)

    return get


def random_checkpoint(spec: LlamaSpec, seed: int = 0, dtype=torch.float32) -> Dict[str, torch.Tensor]:
    src = random_source(spec, seed, "cpu", dtype)
    return {n: src(n) for n, _ in checkpoint_names(spec)}


# ---------------------------------------------------------------------------
# Runtime layout
# ---------------------------------------------------------------------------
@dataclasses.dataclass
class LayerWeights:
    ln1: torch.Tensor
    wqkv: torch.Tensor
    wo: torch.Tensor
    ln2: torch.Tensor
    wgu: Optional[torch.Tensor] = None       # dense MLP (interleaved gate/up)
    wd: Optional[torch.Tensor] = None
    router: Optional[torch.Tensor] = None    # MoE [E, H]
    experts_gu: Optional[torch.Tensor] = None  # [E_local, 2F, H] interleaved
    experts_d: Optional[torch.Tensor] = None   # [E_local, H, F]
    # fp8 block-scaled variants (e4m3 weight + fp32 [out/128, in/128] scales)
    fp8: Optional[Dict[str, Tuple[torch.Tensor, torch.Tensor]]] = None


@dataclasses.dataclass
class ModelWeights:
    spec: LlamaSpec
    shard: TPShard
    embed: torch.Tensor
    layers: List[LayerWeights]
    norm: torch.Tensor
    lm_head: torch.Tensor                      # [V / tp, H]
    ep_rank: int = 0                           # expert-parallel position (MoE)
    ep_size: int = 1

    def nbytes(self) -> int:
        n = self.embed.nbytes + self.norm.nbytes + self.lm_head.nbytes
        for l in self.layers:
            for f in dataclasses.fields(l):
                v = getattr(l, f.name)
                if isinstance(v, torch.Tensor):
                    n += v.nbytes
                elif isinstance(v, dict):          # fp8: (e4m3 weight, fp32 block scales)
                    n += sum(t.nbytes for pair in v.values() for t in pair)
        return n


def pad_rows(t: torch.Tensor, rows: int) -> torch.Tensor:
    if t.shape[0] == rows:
        return t
    return torch.cat([t, t.new_zeros((rows - t.shape[0],) + tuple(t.shape[1:]))], 0)


def pad_cols(t: torch.Tensor, cols: int) -> torch.Tensor:
    if t.shape[1] == cols:
        return t
    return torch.cat([t, t.new_zeros((t.shape[0], cols - t.shape[1]))], 1)


def interleave_gate_up(gate: torch.Tensor, up: torch.Tensor, group: int = SWIGLU_GROUP) -> torch.Tensor:
    Fp = -(-gate.shape[0] // group) * group
    gate, up = pad_rows(gate, Fp), pad_rows(up, Fp)
    F, H = gate.shape
    assert F % group == 0, "ffn shard must be a multiple of the interleave group"
    return torch.stack([gate.reshape(F // group, group, H), up.reshape(F // group, group, H)], 1).reshape(2 * F, H)


def deinterleave_gate_up(wgu: torch.Tensor, group: int = SWIGLU_GROUP):
    F2, H = wgu.shape
    v = wgu.reshape(F2 // (2 * group), 2, group, H)
    return v[:, 0].reshape(-1, H), v[:, 1].reshape(-1, H)


def build_runtime(spec: LlamaSpec, source: Source, shard: Optional[TPShard] = None, device="cpu",
                  dtype: Optional[torch.dtype] = None, ep_rank: int = 0, ep_size: int = 1) -> ModelWeights:
    """Streams a checkpoint (``source(name) -> tensor``) into this rank's runtime layout.

    Only this rank's slices are kept on ``device``; no rank materialises the
    whole model (the reference's sharded-materialisation plan,
    docs/PLAN.md:689-699).
    """
    shard = shard or TPShard(0, 1, spec)
    if dtype is None:
        dtype = torch.bfloat16 if spec.dtype == "bf16" else torch.float32
    D = spec.head_dim

    def get(name):
        # the source's own tensor (a zero-copy view of a memory-mapped file for
        # checkpoints): slicing it first means only this rank's bytes are read
        return source(name)

    def dev(t, dt=None):
        # always a copy: the runtime weights never alias the source (a mapped file)
        return t.to(device=device, dtype=dt or dtype, copy=True).contiguous()

    def rows(t, r):
        return t[r.start:r.stop]

    hr = shard.head_range
    kr = shard.kv_head_range
    fr = shard.ffn_range
    layers = []
    for i in range(spec.layers):
        p = layer_prefix(i)
        q = dev(get(p + "self_attn.q_proj.weight")[hr.start * D:hr.stop * D])
        k = dev(get(p + "self_attn.k_proj.weight")[kr.start * D:kr.stop * D])
        v = dev(get(p + "self_attn.v_proj.weight")[kr.start * D:kr.stop * D])
        wqkv = torch.cat([q, k, v], 0).contiguous()
        wo = dev(get(p + "self_attn.o_proj.weight")[:, hr.start * D:hr.stop * D])
        lw = LayerWeights(ln1=dev(get(p + "input_layernorm.weight")), wqkv=wqkv, wo=wo,
                          ln2=dev(get(p + "post_attention_layernorm.weight")))
        if spec.is_moe:
            lw.router = dev(get(p + "block_sparse_moe.gate.weight"), torch.float32)
            e_per = spec.experts // ep_size
            gus, ds = [], []
            for e in range(ep_rank * e_per, (ep_rank + 1) * e_per):
                qq = p + f"block_sparse_moe.experts.{e}."
                g = get(qq + "w1.weight")
                u = get(qq + "w3.weight")
                d = get(qq + "w2.weight")
                if ep_size == 1:
                    g, u, d = rows(g, fr), rows(u, fr), d[:, fr.start:fr.stop]
                gus.append(interleave_gate_up(dev(g), dev(u)))
                ds.append(pad_cols(dev(d), -(-d.shape[1] // SWIGLU_GROUP) * SWIGLU_GROUP))
            lw.experts_gu = torch.stack(gus).contiguous()
            lw.experts_d = torch.stack(ds).contiguous()
        else:
            g = dev(rows(get(p + "mlp.gate_proj.weight"), fr))
            u = dev(rows(get(p + "mlp.up_proj.weight"), fr))
            lw.wgu = interleave_gate_up(g, u).contiguous()
            lw.wd = pad_cols(dev(get(p + "mlp.down_proj.weight")[:, fr.start:fr.stop]), shard.ffn_padded).contiguous()
        if spec.fp8_block and not spec.is_moe:
            # Block-scaled fp8 projections: quantise in the runtime layout (after
            # sharding and the gate/up interleave) and drop the bf16 copies.
            from .fp8 import quantize_weight
            lw.fp8 = {}
            for name in ("wqkv", "wo", "wgu", "wd"):
                lw.fp8[name] = quantize_weight(getattr(lw, name))
                setattr(lw, name, None)
        layers.append(lw)
    embed = dev(get("model.embed_tokens.weight"))
    head_name = "model.embed_tokens.weight" if spec.tie_embeddings else "lm_head.weight"
    vr = shard.vocab_range
    lm_head = dev(get(head_name)[vr.start:vr.stop])
    return ModelWeights(spec=spec, shard=shard, embed=embed, layers=layers,
                        norm=dev(get("model.norm.weight")), lm_head=lm_head,
                        ep_rank=ep_rank, ep_size=ep_size)
