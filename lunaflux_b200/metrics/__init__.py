"""Serving metrics: counters, gauges and fixed-bucket histograms with bounded
label sets, a Prometheus text rendering and a JSON snapshot.

Reference: the metric set is specified in docs/ARCHITECTURE.md:496-511 and
docs/BENCHMARKING.md:53-66 (TTFT and ITL distributions; queue, prefill and
decode times; tokens per step; KV pages free / active / cached / hit /
evicted; failures; graph-capture time) but no metrics package exists there
(README.mbt.md:76-99).  Labels are closed enumerations (finish reason, public
error code, step kind), never request text or ids, so the output carries no
payload and its cardinality is bounded.
"""
from __future__ import annotations

import bisect
import math
import threading
from typing import Dict, Iterable, List, Optional, Sequence, Tuple

# Latency buckets in seconds: 1 ms .. 60 s, roughly x2 apart.
LATENCY_BUCKETS = (0.001, 0.002, 0.005, 0.01, 0.02, 0.05, 0.1, 0.2, 0.5, 1.0, 2.0, 5.0, 10.0, 30.0, 60.0)
COUNT_BUCKETS = (1, 2, 4, 8, 16, 32, 64, 128, 256, 512, 1024, 2048, 4096, 8192, 16384)
MAX_LABEL_VALUES = 64


class MetricError(ValueError):
    pass


class _Metric:
    kind = ""

    def __init__(self, name: str, help_: str, labels: Sequence[str] = ()):
        if not name.replace("_", "").isalnum():
            raise MetricError(f"bad metric name {name!r}")
        self.name, self.help, self.labels = name, help_, tuple(labels)
        self._lock = threading.Lock()

    def _key(self, labels: Dict[str, str]) -> Tuple[str, ...]:
        if set(labels) != set(self.labels):
            raise MetricError(f"{self.name}: labels {sorted(labels)} != {sorted(self.labels)}")
        return tuple(str(labels[k]) for k in self.labels)

    def _fmt_labels(self, key: Tuple[str, ...], extra: str = "") -> str:
        parts = [f'{k}="{v}"' for k, v in zip(self.labels, key)]
        if extra:
            parts.append(extra)
        return "{" + ",".join(parts) + "}" if parts else ""


class Counter(_Metric):
    kind = "counter"

    def __init__(self, name, help_, labels=()):
        super().__init__(name, help_, labels)
        self.values: Dict[Tuple[str, ...], float] = {}

    def inc(self, amount: float = 1.0, **labels):
        if amount < 0:
            raise MetricError("counters only go up")
        k = self._key(labels)
        with self._lock:
            if k not in self.values and len(self.values) >= MAX_LABEL_VALUES:
                raise MetricError(f"{self.name}: label cardinality limit")
            self.values[k] = self.values.get(k, 0.0) + amount

    def get(self, **labels) -> float:
        return self.values.get(self._key(labels), 0.0)

    def render(self) -> List[str]:
        return [f"{self.name}{self._fmt_labels(k)} {_num(v)}" for k, v in sorted(self.values.items())]

    def snapshot(self):
        return {",".join(k) or "": v for k, v in self.values.items()}


class Gauge(Counter):
    kind = "gauge"

    def set(self, value: float, **labels):
        k = self._key(labels)
        with self._lock:
            if k not in self.values and len(self.values) >= MAX_LABEL_VALUES:
                raise MetricError(f"{self.name}: label cardinality limit")
            self.values[k] = float(value)


class Histogram(_Metric):
    kind = "histogram"

    def __init__(self, name, help_, buckets: Sequence[float] = LATENCY_BUCKETS, labels=()):
        super().__init__(name, help_, labels)
        if list(buckets) != sorted(buckets) or not buckets:
            raise MetricError("buckets must be increasing")
        self.buckets = tuple(float(b) for b in buckets)
        self.series: Dict[Tuple[str, ...], List[float]] = {}   # [count per bucket..., +Inf, sum, n]

    def observe(self, value: float, **labels):
        if value is None or math.isnan(value):
            return
        k = self._key(labels)
        with self._lock:
            s = self.series.get(k)
            if s is None:
                if len(self.series) >= MAX_LABEL_VALUES:
                    raise MetricError(f"{self.name}: label cardinality limit")
                s = self.series[k] = [0.0] * (len(self.buckets) + 3)
            s[bisect.bisect_left(self.buckets, value)] += 1
            s[-2] += value
            s[-1] += 1

    def count(self, **labels) -> int:
        s = self.series.get(self._key(labels))
        return int(s[-1]) if s else 0

    def quantile(self, q: float, **labels) -> Optional[float]:
        """Upper bucket bound below which a fraction q of observations fall."""
        s = self.series.get(self._key(labels))
        if not s or s[-1] == 0:
            return None
        target, run = q * s[-1], 0.0
        for i, b in enumerate(self.buckets):
            run += s[i]
            if run >= target:
                return b
        return math.inf

    def render(self) -> List[str]:
        out = []
        for k, s in sorted(self.series.items()):
            run = 0.0
            for i, b in enumerate(self.buckets):
                run += s[i]
                out.append(f"{self.name}_bucket{self._fmt_labels(k, f'le=\"{_num(b)}\"')} {_num(run)}")
            out.append(f"{self.name}_bucket{self._fmt_labels(k, 'le=\"+Inf\"')} {_num(s[-1])}")
            out.append(f"{self.name}_sum{self._fmt_labels(k)} {_num(s[-2])}")
            out.append(f"{self.name}_count{self._fmt_labels(k)} {_num(s[-1])}")
        return out

    def snapshot(self):
        return {",".join(k) or "": {"count": int(s[-1]), "sum": s[-2], "p50": self.quantile(0.5, **dict(zip(self.labels, k))),
                                     "p99": self.quantile(0.99, **dict(zip(self.labels, k)))}
                for k, s in self.series.items()}


def _num(v: float) -> str:
    return repr(int(v)) if float(v).is_integer() else repr(float(v))


class Registry:
    def __init__(self):
        self.metrics: Dict[str, _Metric] = {}

    def _add(self, m):
        if m.name in self.metrics:
            raise MetricError(f"duplicate metric {m.name}")
        self.metrics[m.name] = m
        return m

    def counter(self, name, help_, labels=()) -> Counter:
        return self._add(Counter(name, help_, labels))

    def gauge(self, name, help_, labels=()) -> Gauge:
        return self._add(Gauge(name, help_, labels))

    def histogram(self, name, help_, buckets=LATENCY_BUCKETS, labels=()) -> Histogram:
        return self._add(Histogram(name, help_, buckets, labels))

    def render_prometheus(self) -> str:
        lines = []
        for m in self.metrics.values():
            lines.append(f"# HELP {m.name} {m.help}")
            lines.append(f"# TYPE {m.name} {m.kind}")
            lines.extend(m.render())
        return "\n".join(lines) + "\n"

    def snapshot(self) -> Dict[str, object]:
        return {n: m.snapshot() for n, m in self.metrics.items()}


class EngineMetrics:
    """The serving metric set, updated by ``LLMEngine``."""

    def __init__(self, registry: Optional[Registry] = None):
        r = self.registry = registry or Registry()
        self.requests = r.counter("lunaflux_requests_total", "Requests admitted")
        self.finished = r.counter("lunaflux_requests_finished_total", "Requests finished, by finish reason",
                                  ("reason",))
        self.failed = r.counter("lunaflux_requests_failed_total", "Requests failed, by public error code", ("code",))
        self.ttft = r.histogram("lunaflux_ttft_seconds", "Arrival to first token")
        self.tpot = r.histogram("lunaflux_tpot_seconds", "Mean time per output token after the first")
        self.itl = r.histogram("lunaflux_itl_seconds", "Time between consecutive engine steps that emitted tokens")
        self.queue = r.histogram("lunaflux_queue_seconds", "Arrival to first scheduled step")
        self.step_time = r.histogram("lunaflux_step_seconds", "Engine step wall time, by kind", labels=("kind",))
        self.step_tokens = r.histogram("lunaflux_step_tokens", "Tokens per engine step", COUNT_BUCKETS)
        self.step_rows = r.histogram("lunaflux_step_rows", "Rows (requests) per engine step", COUNT_BUCKETS)
        self.output_tokens = r.counter("lunaflux_output_tokens_total", "Generated tokens")
        self.prompt_tokens = r.counter("lunaflux_prompt_tokens_total", "Prompt tokens of finished requests")
        self.cached_tokens = r.counter("lunaflux_prefix_cached_tokens_total", "Prompt tokens served by the prefix cache")
        self.kv_pages = r.gauge("lunaflux_kv_pages", "KV pages by state", ("state",))
        self.graph = r.counter("lunaflux_graph_steps_total", "Steps by execution mode", ("mode",))
        self.graph_capture = r.histogram("lunaflux_graph_capture_seconds", "CUDA-graph capture time")
        self._last_emit: Optional[float] = None

    def prefix_hit_rate(self) -> Optional[float]:
        p = self.prompt_tokens.get()
        return None if p == 0 else self.cached_tokens.get() / p
