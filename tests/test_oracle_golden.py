"""The fp32 oracle operators against the reference's golden values
(kernels/reference/operations_test.mbt: RMSNorm, split-half RoPE, causal GQA,
SiLU-gated MLP), computed by the reference outside this repository."""
import math

import torch

from lunaflux_b200.oracle.reference import causal_gqa_attention, rms_norm, rope_angles, rotary, silu_gated_mlp


def close(got, want, tol):
    got = [float(x) for x in torch.as_tensor(got).reshape(-1)]
    assert len(got) == len(want) and all(abs(a - b) <= tol for a, b in zip(got, want)), (got, want)


def test_rms_norm_golden():
    close(rms_norm(torch.tensor([[3.0, 4.0]]), torch.ones(2), 1e-5), [0.8485277, 1.1313703], 2e-5)


def test_split_half_rope_golden():
    cos, sin = rope_angles(torch.tensor([1]), 4, 10000.0, dtype=torch.float32)
    q = torch.tensor([[[1.0, 2.0, 3.0, 4.0]]])
    k = torch.tensor([[[5.0, 6.0, 7.0, 8.0]]])
    close(rotary(q, cos, sin), [-1.9841106, 1.9599007, 2.4623778, 4.0197997], 3e-5)
    close(rotary(k, cos, sin), [-3.1887856, 5.919701, 7.9894705, 8.059599], 3e-5)
    cos, sin = rope_angles(torch.tensor([1]), 2, 10000.0, dtype=torch.float32)
    close(rotary(torch.tensor([[[1.0, 0.0]]]), cos, sin), [0.5403023, 0.8414710], 2e-5)
    close(rotary(torch.tensor([[[0.0, 1.0]]]), cos, sin), [-0.8414710, 0.5403023], 2e-5)


def test_causal_gqa_golden():
    q = torch.zeros(2, 2, 2)
    k = torch.zeros(2, 1, 2)
    v = torch.tensor([[[2.0, 4.0]], [[4.0, 8.0]]])
    close(causal_gqa_attention(q, k, v, 1 / math.sqrt(2)), [2, 4, 2, 4, 3, 6, 3, 6], 1e-6)


def test_silu_gated_mlp_golden():
    one = torch.tensor([[1.0]])
    close(silu_gated_mlp(one, torch.tensor([[1.0]]), torch.tensor([[2.0]]), torch.tensor([[3.0]])), [4.3863516], 2e-5)
