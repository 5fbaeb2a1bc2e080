"""Block-scaled fp8 (e4m3) weights and activations.

Weights: one fp32 scale per 128 x 128 block, ``scale = amax / 448`` and
``w8 = w / scale`` rounded to e4m3 (the layout of DeepSeek-style fp8
checkpoints, ``*.weight`` e4m3 + ``*.weight_scale_inv`` fp32).  Activations:
one scale per token per 128 channels, produced on the device by the
``act_quant`` kernel right before each projection.
"""
from __future__ import annotations

from typing import Tuple

import torch

E4M3_MAX = 448.0
BLOCK = 128


def quantize_weight(w: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """[N, K] -> (e4m3 [N, K], fp32 scales [ceil(N/128), K/128])."""
    N, K = w.shape
    if K % BLOCK:
        raise ValueError("fp8 weights need K % 128 == 0")
    Np = -(-N // BLOCK) * BLOCK
    wf = w.float()
    if Np != N:
        wf = torch.cat([wf, wf.new_zeros(Np - N, K)], 0)
    blocks = wf.view(Np // BLOCK, BLOCK, K // BLOCK, BLOCK)
    amax = blocks.abs().amax(dim=(1, 3)).clamp_min(1e-12)
    scale = amax / E4M3_MAX
    q = (blocks / scale[:, None, :, None]).clamp(-E4M3_MAX, E4M3_MAX).view(Np, K)[:N]
    return q.to(torch.float8_e4m3fn).contiguous(), scale.contiguous()


def dequantize_weight(q: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    N, K = q.shape
    s = scale.repeat_interleave(BLOCK, 0)[:N].repeat_interleave(BLOCK, 1)
    return q.float() * s


def quantize_act(x: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """Reference per-token, per-128-channel quantisation (same rule as the kernel)."""
    M, K = x.shape
    xb = x.float().view(M, K // BLOCK, BLOCK)
    scale = xb.abs().amax(-1).clamp_min(1e-12) / E4M3_MAX
    q = (xb / scale[..., None]).view(M, K).to(torch.float8_e4m3fn)
    return q, scale
