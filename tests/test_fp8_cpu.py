"""Block-scaled fp8 projections through the engine (CPU operator set)."""
import torch

from lunaflux_b200.config import CacheConfig, SchedulerConfig
from lunaflux_b200.engine.engine import EngineOptions, LLMEngine
from lunaflux_b200.models.fp8 import dequantize_weight, quantize_act, quantize_weight
from lunaflux_b200.models.spec import LlamaSpec
from lunaflux_b200.models.weights import build_runtime, random_checkpoint
from lunaflux_b200.ops.torch_ops import TorchOps
from lunaflux_b200.oracle.reference import ReferenceModel


def test_weight_quantisation_error_is_small():
    w = torch.randn(300, 512) * 0.02
    q, s = quantize_weight(w)
    assert q.dtype == torch.float8_e4m3fn and s.shape == (3, 4)
    err = (dequantize_weight(q, s) - w).abs().max() / w.abs().max()
    assert err < 0.07
    x = torch.randn(5, 256)
    qa, sa = quantize_act(x)
    assert ((qa.float() * sa.repeat_interleave(128, 1)) - x).abs().max() / x.abs().max() < 0.07


def test_fp8_engine_tracks_the_oracle():
    spec = LlamaSpec(hidden=128, layers=2, heads=2, kv_heads=1, head_dim=64, ffn=128, vocab=256, max_position=512,
                     dtype="fp32", fp8_block=128)
    ck = random_checkpoint(spec, 0, dtype=torch.float32)
    ck = {k: v * 5 if v.dim() == 2 else v for k, v in ck.items()}  # larger weights: sharper logits
    w = build_runtime(spec, lambda n: ck[n])
    assert w.layers[0].fp8 is not None and w.layers[0].wqkv is None
    eng = LLMEngine(w, TorchOps(), "cpu", SchedulerConfig(step_token_budget=64, max_active_requests=4,
                                                          prefill_chunk_tokens=64, emergency_decode_page_reserve=1),
                    CacheConfig(), EngineOptions(max_context=256, num_pages=64, graph_sizes=()))
    g = torch.Generator().manual_seed(1)
    prompts = [torch.randint(0, 256, (n,), generator=g).tolist() for n in (6, 20)]
    outs = eng.generate(prompts, 6)
    ref = ReferenceModel(spec, ck)
    for p, o in zip(prompts, outs):
        logits = ref.forward(list(p) + o)
        for i, tok in enumerate(o):
            row = logits[len(p) - 1 + i]
            assert (row.max() - row[tok]).item() <= 0.25 * row.std().item()
