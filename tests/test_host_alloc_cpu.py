"""Host-side allocation budget of the steady decode step (scheduler, step
packing, sampling readback, commit), measured with tracemalloc on the CPU
engine.  Reference: tests/hot_path_alloc (every allocation in the warm step
window is counted; the budget there is zero allocations).  A Python control
path cannot reach zero object churn, so the gates are: no net growth of the
Python heap across a long window of steady steps beyond the tokens it
records, and a bounded transient peak per step."""
import tracemalloc

import torch

from lunaflux_b200.config import CacheConfig, SchedulerConfig
from lunaflux_b200.engine.engine import EngineOptions, LLMEngine
from lunaflux_b200.models.spec import tiny_llama
from lunaflux_b200.models.weights import build_runtime, random_checkpoint
from lunaflux_b200.ops.torch_ops import TorchOps

STEPS = 120
# Measured (CPU, 16 decoding requests, 120 steps): net growth about 75 KB: the
# 16 output token lists, the page ids of pages the growing sequences take, and
# interpreter free-lists that plateau; per-step transient peak about 15 KB.
NET_BUDGET_BYTES = 160 * 1024         # over the whole window
PEAK_BUDGET_BYTES = 64 * 1024         # transient Python heap above the step's starting level


def _engine(overlap):
    spec = tiny_llama()
    ck = random_checkpoint(spec, 0)
    return LLMEngine(build_runtime(spec, lambda n: ck[n]), TorchOps(), "cpu",
                     SchedulerConfig(step_token_budget=256, max_active_requests=16, prefill_chunk_tokens=256,
                                     emergency_decode_page_reserve=4),
                     CacheConfig(prefix_enabled=False),
                     EngineOptions(max_context=512, num_pages=600, graph_sizes=(), overlap_steps=overlap))


def _measure(overlap):
    eng = _engine(overlap)
    g = torch.Generator().manual_seed(0)
    for _ in range(16):
        eng.add_request(torch.randint(0, 256, (12,), generator=g).tolist(), STEPS + 60)
    for _ in range(30):                       # prefill and warm decode steps
        eng.step()
    assert all(r.num_computed >= len(r.prompt) for r in eng.live.values())
    tracemalloc.start()
    try:
        base, _ = tracemalloc.get_traced_memory()
        worst = 0
        for _ in range(STEPS):
            tracemalloc.reset_peak()
            start, _ = tracemalloc.get_traced_memory()
            assert eng.step()
            _, peak = tracemalloc.get_traced_memory()
            worst = max(worst, peak - start)
        end, _ = tracemalloc.get_traced_memory()
    finally:
        tracemalloc.stop()
    return end - base, worst


def test_steady_decode_host_allocation_budget():
    for overlap in (False, True):
        net, worst = _measure(overlap)
        assert net <= NET_BUDGET_BYTES, f"overlap={overlap}: Python heap grew by {net} bytes over {STEPS} steps"
        assert worst <= PEAK_BUDGET_BYTES, f"overlap={overlap}: a step's transient peak was {worst} bytes"
