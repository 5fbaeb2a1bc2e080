"""Metrics registry and the engine's serving metrics (CPU, config #1 model)."""
import math

import pytest

from lunaflux_b200.metrics import Counter, EngineMetrics, Histogram, MetricError, Registry


def test_registry_render_and_limits():
    r = Registry()
    c = r.counter("x_total", "things", ("kind",))
    h = r.histogram("lat_seconds", "latency", (0.1, 1.0))
    g = r.gauge("level", "a level")
    c.inc(kind="a")
    c.inc(2, kind="b")
    h.observe(0.05)
    h.observe(0.5)
    h.observe(5.0)
    g.set(3)
    text = r.render_prometheus()
    assert 'x_total{kind="a"} 1' in text and 'x_total{kind="b"} 2' in text
    assert 'lat_seconds_bucket{le="0.1"} 1' in text and 'lat_seconds_bucket{le="1"} 2' in text
    assert 'lat_seconds_bucket{le="+Inf"} 3' in text and "lat_seconds_count 3" in text
    assert "level 3" in text
    assert h.quantile(0.5) == 1.0 and h.quantile(1.0) == math.inf
    with pytest.raises(MetricError):
        c.inc(-1, kind="a")
    with pytest.raises(MetricError):
        c.inc(other="a")
    with pytest.raises(MetricError):
        r.counter("x_total", "dup")
    many = Counter("m_total", "", ("k",))
    for i in range(64):
        many.inc(k=str(i))
    with pytest.raises(MetricError):
        many.inc(k="one too many")
    assert isinstance(r.snapshot()["lat_seconds"][""]["count"], int)


def test_engine_updates_metrics():
    import torch

    from lunaflux_b200.config import CacheConfig, SchedulerConfig
    from lunaflux_b200.engine.engine import EngineOptions, LLMEngine
    from lunaflux_b200.models.spec import tiny_llama
    from lunaflux_b200.models.weights import build_runtime, random_source
    from lunaflux_b200.ops.torch_ops import TorchOps
    spec = tiny_llama()
    w = build_runtime(spec, random_source(spec, seed=1), device="cpu", dtype=torch.float32)
    eng = LLMEngine(w, TorchOps(), "cpu", SchedulerConfig(), CacheConfig(),
                    EngineOptions(max_context=256, num_pages=64, graph_sizes=()))
    prompt = list(range(3, 40))
    eng.generate([prompt, prompt], 5)
    eng.generate([prompt], 3)          # the second time the prompt's full pages hit the prefix cache
    m: EngineMetrics = eng.metrics
    assert m.requests.get() == 3
    assert m.finished.get(reason="token_limit") == 3
    assert m.output_tokens.get() == 13
    assert m.ttft.count() == 3 and m.tpot.count() == 3
    assert m.cached_tokens.get() > 0 and 0 < m.prefix_hit_rate() < 1
    assert m.step_time.count(kind="prefill") >= 1 and m.step_time.count(kind="decode") >= 1
    assert m.graph.get(mode="eager") >= 1
    assert m.kv_pages.get(state="free") + m.kv_pages.get(state="allocated") > 0
    assert "lunaflux_ttft_seconds_count 3" in m.registry.render_prometheus()


def test_bench_serving_summary_reads_the_engine_metrics():
    """bench.py's serving block (queue time, tokens per step, graph capture,
    prefix hit rate, finish / failure counts) from a populated metric set and
    from an empty one."""
    import importlib.util
    import os
    from lunaflux_b200.metrics import EngineMetrics
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    spec = importlib.util.spec_from_file_location("lf_bench", os.path.join(root, "bench.py"))
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    m = EngineMetrics()
    for v in (0.001, 0.002, 0.2):
        m.queue.observe(v)
    for t in (256, 8192):
        m.step_tokens.observe(t)
        m.step_rows.observe(8)
    m.graph.inc(mode="captured")
    m.graph.inc(mode="captured")
    m.graph.inc(mode="eager")
    m.graph_capture.observe(0.25)
    m.prompt_tokens.inc(100)
    m.cached_tokens.inc(25)
    m.finished.inc(reason="token_limit")
    m.failed.inc(code="deadline_exceeded")
    s = bench.serving_summary(m)
    assert s["tokens_per_step_mean"] == 4224.0 and s["rows_per_step_mean"] == 8.0
    assert s["graph_captures"] == 1 and s["graph_capture_s"] == 0.25 and s["graph_step_share"] == round(2 / 3, 4)
    assert s["prefix_hit_rate"] == 0.25
    assert s["queue_p50_ms_le"] >= 2.0 and s["queue_p99_ms_le"] >= 200.0
    assert s["finished"] == {"token_limit": 1} and s["failed"] == {"deadline_exceeded": 1}
    empty = bench.serving_summary(EngineMetrics())
    assert empty["tokens_per_step_mean"] is None and empty["finished"] == {}
