"""CPU numerical oracle: an unpaged, full-recompute Llama / Mixtral forward.

A float32 (optionally float64) restatement of the reference's CPU kernels
(kernels/reference/basic.mbt:3-181, rotary.mbt:187-243, attention.mbt:251-330,
mlp.mbt:335-369) and of its greedy full-recompute generator
(engine/reference/generate.mbt): every step re-runs the whole sequence with no
KV cache and takes the argmax of the last row.  It is the ground truth that
the paged engine and every GPU kernel are tested against.
"""
from __future__ import annotations

import math
from typing import Dict, List, Sequence

import torch

from ..models.spec import LlamaSpec, rope_inv_freq
from ..models.weights import checkpoint_names, layer_prefix


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w


def rope_angles(positions: torch.Tensor, head_dim: int, theta: float, dtype=torch.float64, scaling: tuple = ()):
    inv = rope_inv_freq(head_dim, theta, scaling)
    ang = positions.to(torch.float64)[:, None] * inv[None, :]
    return ang.cos().to(dtype), ang.sin().to(dtype)


def rotary(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """Split-half rotation: x [T, heads, D]; angle[i] = pos / theta^(2i/D)."""
    d = x.shape[-1] // 2
    x1, x2 = x[..., :d], x[..., d:]
    c, s = cos[:, None, :], sin[:, None, :]
    return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], -1)


def causal_gqa_attention(q, k, v, scale: float) -> torch.Tensor:
    """q [T, Hq, D], k/v [T, Hkv, D]; contiguous query-head groups per KV head."""
    T, Hq, D = q.shape
    G = Hq // k.shape[1]
    k = k.repeat_interleave(G, 1)
    v = v.repeat_interleave(G, 1)
    s = torch.einsum("thd,uhd->htu", q, k) * scale
    mask = torch.ones(T, T, dtype=torch.bool).triu(1)
    s = s.masked_fill(mask[None], float("-inf"))
    s = s - s.amax(-1, keepdim=True)
    p = s.exp()
    p = p / p.sum(-1, keepdim=True)
    return torch.einsum("htu,uhd->thd", p, v)


def silu_gated_mlp(x, wg, wu, wd):
    g = x @ wg.t()
    return (g * torch.sigmoid(g) * (x @ wu.t())) @ wd.t()


def moe_mlp(x, router, experts, top_k: int):
    """Mixtral MoE: softmax over router logits, top-k experts, renormalised."""
    logits = x @ router.t()
    probs = logits.softmax(-1)
    w, idx = probs.topk(top_k, -1)
    w = w / w.sum(-1, keepdim=True)
    out = torch.zeros_like(x)
    for e, (wg, wu, wd) in enumerate(experts):
        sel = (idx == e)
        rows = sel.any(-1).nonzero().flatten()
        if rows.numel() == 0:
            continue
        we = (w * sel).sum(-1)[rows]
        out[rows] += we[:, None] * silu_gated_mlp(x[rows], wg, wu, wd)
    return out


class ReferenceModel:
    """Holds a checkpoint (HF names) in float32/float64 on the CPU."""

    def __init__(self, spec: LlamaSpec, tensors: Dict[str, torch.Tensor], dtype=torch.float32):
        self.spec = spec
        self.dtype = dtype
        self.t = {n: tensors[n].to(dtype) for n, _ in checkpoint_names(spec)}

    def forward(self, tokens: Sequence[int]) -> torch.Tensor:
        """Logits [T, V] for a full sequence (positions 0..T-1)."""
        s, t = self.spec, self.t
        ids = torch.tensor(list(tokens), dtype=torch.long)
        x = t["model.embed_tokens.weight"][ids]
        T = x.shape[0]
        cos, sin = rope_angles(torch.arange(T), s.head_dim, s.rope_theta, self.dtype, s.rope_scaling)
        scale = 1.0 / math.sqrt(s.head_dim)
        for i in range(s.layers):
            p = layer_prefix(i)
            h = rms_norm(x, t[p + "input_layernorm.weight"], s.rms_eps)
            q = (h @ t[p + "self_attn.q_proj.weight"].t()).view(T, s.heads, s.head_dim)
            k = (h @ t[p + "self_attn.k_proj.weight"].t()).view(T, s.kv_heads, s.head_dim)
            v = (h @ t[p + "self_attn.v_proj.weight"].t()).view(T, s.kv_heads, s.head_dim)
            q, k = rotary(q, cos, sin), rotary(k, cos, sin)
            a = causal_gqa_attention(q, k, v, scale).reshape(T, s.q_size)
            x = x + a @ t[p + "self_attn.o_proj.weight"].t()
            h = rms_norm(x, t[p + "post_attention_layernorm.weight"], s.rms_eps)
            if s.is_moe:
                experts = [(t[p + f"block_sparse_moe.experts.{e}.w1.weight"],
                            t[p + f"block_sparse_moe.experts.{e}.w3.weight"],
                            t[p + f"block_sparse_moe.experts.{e}.w2.weight"]) for e in range(s.experts)]
                x = x + moe_mlp(h, t[p + "block_sparse_moe.gate.weight"], experts, s.experts_per_token)
            else:
                x = x + silu_gated_mlp(h, t[p + "mlp.gate_proj.weight"], t[p + "mlp.up_proj.weight"],
                                       t[p + "mlp.down_proj.weight"])
        x = rms_norm(x, t["model.norm.weight"], s.rms_eps)
        head = t["model.embed_tokens.weight"] if s.tie_embeddings else t["lm_head.weight"]
        return x @ head.t()

    def generate_greedy(self, prompt: Sequence[int], max_new: int) -> List[int]:
        """Greedy full-recompute loop (engine/reference/generate.mbt)."""
        seq = list(prompt)
        out = []
        for _ in range(max_new):
            logits = self.forward(seq)[-1]
            tok = greedy(logits)
            out.append(tok)
            seq.append(tok)
        return out


def greedy(logits: torch.Tensor) -> int:
    """Max finite logit, lowest token id on ties (sampling/greedy.mbt)."""
    if not torch.isfinite(logits).all():
        raise ValueError("non-finite logit")
    m = logits.max()
    return int((logits == m).nonzero()[0].item())
