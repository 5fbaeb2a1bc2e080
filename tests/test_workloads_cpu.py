"""Benchmark workload generators and the workload driver (CPU, tiny model)."""
import numpy as np
import pytest

from lunaflux_b200.bench import workloads as W
from lunaflux_b200.config import CacheConfig, SchedulerConfig
from lunaflux_b200.contracts import SamplingParameters
from lunaflux_b200.engine.engine import EngineOptions, LLMEngine
from lunaflux_b200.models.spec import tiny_llama
from lunaflux_b200.models.weights import build_runtime, random_checkpoint
from lunaflux_b200.ops.torch_ops import TorchOps


def test_generators_match_the_named_configs():
    c2 = W.config2()
    assert len(c2.items) == 256 and all(len(i.prompt) == 1024 and i.max_new == 256 for i in c2.items)
    c3 = W.config3()
    assert len(c3.items) == 128 and c3.items[0].sampling.top_p == 0.9 and c3.items[0].sampling.temperature == 0.7
    assert len({i.sampling.seed for i in c3.items}) == 128
    c4 = W.config4()
    assert len(c4.items) == 512 and c4.router_zipf == 0.5 and max(int(i.prompt.max()) for i in c4.items) < 32000
    c5 = W.config5()
    assert len(c5.items) == 1024
    arr = np.array([i.arrival for i in c5.items])
    assert np.all(np.diff(arr) > 0) and abs(1024 / arr[-1] - 40) < 5
    assert 0.02 < np.mean([i.cancel_after is not None for i in c5.items]) < 0.09
    assert all(2048 + 64 <= len(i.prompt) <= 2048 + 512 and 32 <= i.max_new <= 256 for i in c5.items)
    b = W.zipf_router_bias(8, 0.5, "cpu")
    assert b[0] > b[7]


@pytest.mark.parametrize("overlap", [False, True])
def test_driver_with_arrivals_cancels_and_prefix_hits(overlap):
    spec = tiny_llama()
    ck = random_checkpoint(spec, 0)
    eng = LLMEngine(build_runtime(spec, lambda n: ck[n]), TorchOps(), "cpu",
                    SchedulerConfig(step_token_budget=64, max_active_requests=4, prefill_chunk_tokens=64,
                                    emergency_decode_page_reserve=1),
                    CacheConfig(), EngineOptions(max_context=256, num_pages=96, graph_sizes=(), overlap_steps=overlap))
    rng = np.random.default_rng(0)
    shared = rng.integers(0, 256, 48, dtype=np.int32)
    items = [W.WorkItem(np.concatenate([shared, rng.integers(0, 256, 5, dtype=np.int32)]), 6, SamplingParameters(),
                        arrival=0.01 * i, cancel_after=3 if i == 2 else None) for i in range(6)]
    ticks = iter(range(1 << 30))
    # a clock that advances 5 ms per reading: arrivals interleave with steps
    # the same way on a loaded machine as on an idle one
    st = W.run(eng, W.Workload("t", "tiny", items, prefix_cache=True), clock=lambda: 0.005 * next(ticks))
    s = st.summary()
    assert s["cancelled"] == 1 and s["finished"] == 5
    assert st.tokens == 5 * 6 + 3
    assert s["prefix_hit_rate"] > 0.3
    assert eng.scheduler.allocator.allocated_page_count() == eng.scheduler.prefix.page_count()
