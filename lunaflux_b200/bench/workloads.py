"""The benchmark workloads of the five named configurations.

Each workload is a list of requests (prompt tokens, output length, sampling,
arrival time, cancellation point) generated from a seed, plus a driver loop
that feeds them to an ``LLMEngine`` and collects per-request timings.  All
ranks of a tensor-parallel group run the same deterministic scheduler; when
arrivals depend on wall time, rank 0 decides how many requests arrive before
each iteration and broadcasts that count, so every rank admits the same ones.

  config 1  tiny-llama CPU plumbing (tests/test_engine_cpu.py)
  config 2  llama3-8b,      256 x (1024 -> 256), greedy, all at t = 0
  config 3  llama3-70b-fp8, 128 x (2048 -> 512), top-p 0.9 at T 0.7, seed 0
  config 4  mixtral-8x7b,   512 x (512 -> 128), greedy, Zipf(0.5)-skewed router
  config 5  llama3-8b prefix/Poisson: 1024 requests at 40 req/s, 4 shared
            2048-token prefixes + 64..512 unique tokens, 32..256 outputs,
            5 % cancelled mid-decode
"""
from __future__ import annotations

import dataclasses
import math
import statistics
import time
from typing import Dict, List, Optional

import numpy as np
import torch

from ..contracts import SamplingParameters, derive_seed


@dataclasses.dataclass
class WorkItem:
    prompt: np.ndarray
    max_new: int
    sampling: SamplingParameters
    arrival: float = 0.0
    cancel_after: Optional[int] = None   # cancel once this many tokens were produced
    cache_scope: bytes = b""


@dataclasses.dataclass
class Workload:
    name: str
    model: str
    items: List[WorkItem]
    prefix_cache: bool = False
    router_zipf: float = 0.0
    note: str = ""


def config2(seed: int = 0, requests: int = 256, prompt: int = 1024, output: int = 256, vocab: int = 128256):
    rng = np.random.default_rng(seed)
    items = [WorkItem(rng.integers(0, vocab, prompt, dtype=np.int32), output, SamplingParameters())
             for _ in range(requests)]
    return Workload("config2", "llama3-8b", items)


def config3(seed: int = 0, requests: int = 128, prompt: int = 2048, output: int = 512, vocab: int = 128256):
    rng = np.random.default_rng(seed)
    items = [WorkItem(rng.integers(0, vocab, prompt, dtype=np.int32), output,
                      SamplingParameters.sample(0.7, top_p=0.9, seed=derive_seed(seed, i))) for i in range(requests)]
    return Workload("config3", "llama3-70b-fp8", items)


def config4(seed: int = 0, requests: int = 512, prompt: int = 512, output: int = 128, vocab: int = 32000):
    rng = np.random.default_rng(seed)
    items = [WorkItem(rng.integers(0, vocab, prompt, dtype=np.int32), output, SamplingParameters())
             for _ in range(requests)]
    return Workload("config4", "mixtral-8x7b", items, router_zipf=0.5)


def config5(seed: int = 0, requests: int = 1024, rate: float = 40.0, vocab: int = 128256, prefixes: int = 4,
            prefix_len: int = 2048, cancel_frac: float = 0.05):
    rng = np.random.default_rng(seed)
    shared = [rng.integers(0, vocab, prefix_len, dtype=np.int32) for _ in range(prefixes)]
    t = 0.0
    items = []
    for i in range(requests):
        t += rng.exponential(1.0 / rate)
        uniq = rng.integers(0, vocab, int(rng.integers(64, 513)), dtype=np.int32)
        out = int(rng.integers(32, 257))
        cancel = int(rng.integers(1, out)) if rng.random() < cancel_frac else None
        items.append(WorkItem(np.concatenate([shared[int(rng.integers(0, prefixes))], uniq]), out,
                              SamplingParameters(), arrival=t, cancel_after=cancel))
    return Workload("config5", "llama3-8b", items, prefix_cache=True)


WORKLOADS = {"config2": config2, "config3": config3, "config4": config4, "config5": config5}


def zipf_router_bias(experts: int, s: float, device) -> torch.Tensor:
    """Logit bias that skews a near-uniform router towards Zipf(s) expert load."""
    p = np.array([1.0 / (e + 1) ** s for e in range(experts)])
    p /= p.sum()
    return torch.tensor(np.log(p * experts), dtype=torch.float32, device=device)


@dataclasses.dataclass
class RunStats:
    tokens: int
    wall_s: float
    ttft_ms: List[float]
    tpot_ms: List[float]
    finished: int
    cancelled: int
    goodput_tokens: int
    prefix_hit_tokens: int
    prompt_tokens: int
    iterations: int

    def summary(self) -> Dict[str, object]:
        def pct(v, q):
            return round(float(np.percentile(v, q)), 3) if v else None
        return {"output_tokens": self.tokens, "wall_s": round(self.wall_s, 3),
                "ttft_p50_ms": pct(self.ttft_ms, 50), "ttft_p99_ms": pct(self.ttft_ms, 99),
                "tpot_p50_ms": pct(self.tpot_ms, 50), "tpot_p99_ms": pct(self.tpot_ms, 99),
                "finished": self.finished, "cancelled": self.cancelled,
                "goodput_tokens_per_s": round(self.goodput_tokens / self.wall_s, 1) if self.wall_s else None,
                "prefix_hit_rate": round(self.prefix_hit_tokens / max(1, self.prompt_tokens), 4),
                "iterations": self.iterations}


def run(engine, wl: Workload, comm=None, realtime: bool = True, clock=time.perf_counter) -> RunStats:
    """Feeds a workload through ``engine`` and returns per-request statistics.
    Requests with arrival > 0 are admitted when ``clock`` reaches them
    (rank 0's clock, broadcast); cancellations happen after the given number
    of produced tokens."""
    import torch.distributed as dist
    engine.results.clear()
    sched = engine.scheduler
    hits0 = sched.prefix_hit_tokens
    pending = sorted(range(len(wl.items)), key=lambda i: wl.items[i].arrival)
    rid_of = {}
    produced: Dict[int, int] = {}
    cancel_at: Dict[int, int] = {}
    t0 = clock()
    nxt = 0
    iters = 0
    prompt_tokens = 0
    count_t = torch.zeros(1, dtype=torch.int64, device=engine.device) if comm is not None else None

    def admit(upto: int):
        nonlocal nxt, prompt_tokens
        while nxt < upto:
            it = wl.items[pending[nxt]]
            rid = engine.add_request(it.prompt, it.max_new, it.sampling, cache_scope=it.cache_scope,
                                     use_prefix_cache=wl.prefix_cache, arrival=t0 + it.arrival)
            rid_of[rid] = pending[nxt]
            produced[rid] = 0
            prompt_tokens += len(it.prompt)
            if it.cancel_after is not None:
                cancel_at[rid] = it.cancel_after
            nxt += 1

    while nxt < len(pending) or engine.has_work():
        now = clock() - t0
        n = nxt
        while n < len(pending) and (not realtime or wl.items[pending[n]].arrival <= now):
            n += 1
        if not engine.has_work() and n == nxt and nxt < len(pending):
            n = nxt + 1  # idle: jump to the next arrival
            if realtime:
                time.sleep(max(0.0, wl.items[pending[nxt]].arrival - now))
        if comm is not None:
            count_t.fill_(n)
            dist.broadcast(count_t, 0)
            n = int(count_t.item())
        admit(n)
        outs = engine.step()
        iters += 1
        for o in outs:
            produced[o.rid] = produced.get(o.rid, 0) + 1
            c = cancel_at.get(o.rid)
            if c is not None and produced[o.rid] >= c and not o.finished:
                engine.cancel(o.rid)
                cancel_at.pop(o.rid)
    wall = clock() - t0
    ttft, tpot = [], []
    toks = good = fin = canc = 0
    for rid, res in engine.results.items():
        toks += len(res.tokens)
        if res.ttft is not None:
            ttft.append(res.ttft * 1e3)
        if res.tpot is not None:
            tpot.append(res.tpot * 1e3)
        if res.reason is not None and res.reason.name == "CANCELLED":
            canc += 1
        elif res.error is None:
            fin += 1
            good += len(res.tokens)
    return RunStats(toks, wall, ttft, tpot, fin, canc, good, sched.prefix_hit_tokens - hits0, prompt_tokens, iters)
