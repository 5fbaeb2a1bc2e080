"""Host cost of one engine step, without a device: scheduler planning, the
packed step block, and the commit of the sampled tokens.

    python -m lunaflux_b200.bench.host [--requests 1024] [--rows 256] [--prompt 2048] [--steps 300]

The engine overlaps this work with the device step (``overlap_steps``), so
it only limits throughput when it exceeds the device time of a step.  The
workload is config 5's scale: ``--requests`` requests queued at once, up to
``--rows`` running, prompts of ``--prompt`` tokens through chunked prefill,
then decode; each line of output is the median and p99 of the three host
phases over the measured steps, split into prefill and decode steps.
"""
from __future__ import annotations

import argparse
import gc
import json
import statistics
import time

import numpy as np

from ..config import CacheConfig, SchedulerConfig
from ..contracts import SamplingParameters
from ..engine.step_inputs import build_host_step, make_layout
from ..runtime.clock import FakeClock
from ..scheduler.scheduler import Request, Scheduler


def run(requests: int, rows: int, prompt: int, output: int, budget: int, steps: int, seed: int = 0):
    P = 16
    max_context = prompt + output + P
    pages = rows * (-(-max_context // P)) + 64
    cfg = SchedulerConfig(step_token_budget=budget, max_active_requests=rows, max_waiting_requests=requests,
                          prefill_chunk_tokens=budget, emergency_decode_page_reserve=min(64, rows),
                          output_event_capacity=max(rows, budget))
    sch = Scheduler(cfg, CacheConfig(prefix_enabled=False), pages, clock=FakeClock(), max_context=max_context)
    rng = np.random.default_rng(seed)
    for rid in range(requests):
        # prompts as the engine stores them: a tuple of ints
        sch.add_request(Request(rid, tuple(rng.integers(0, 128000, prompt).tolist()), output, SamplingParameters()))
    W = -(-max_context // P)
    out = np.zeros(make_layout(budget + rows, rows, rows, rows, W).total + 64, dtype=np.int32)
    times = {"prefill": {"plan": [], "pack": [], "commit": []}, "decode": {"plan": [], "pack": [], "commit": []}}
    for _ in range(steps):
        t0 = time.perf_counter()
        plan = sch.schedule()
        if plan is None:
            break
        t1 = time.perf_counter()
        build_host_step(plan, sch.tables.matrix, P, W, out)
        t2 = time.perf_counter()
        sch.complete(plan, rng.integers(0, 128000, len(plan.sample_rows)).tolist())
        t3 = time.perf_counter()
        kind = "prefill" if plan.prefill_rows else "decode"
        for k, v in (("plan", t1 - t0), ("pack", t2 - t1), ("commit", t3 - t2)):
            times[kind][k].append(v * 1e3)
    result = {}
    for kind, phases in times.items():
        if not phases["plan"]:
            continue
        result[kind] = {"steps": len(phases["plan"])}
        for k, v in phases.items():
            v = sorted(v)
            result[kind][f"{k}_p50_ms"] = round(statistics.median(v), 3)
            result[kind][f"{k}_p99_ms"] = round(v[min(len(v) - 1, int(0.99 * len(v)))], 3)
            result[kind][f"{k}_max_ms"] = round(v[-1], 3)
    return result


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--requests", type=int, default=1024)
    ap.add_argument("--rows", type=int, default=256)
    ap.add_argument("--prompt", type=int, default=2048)
    ap.add_argument("--output", type=int, default=256)
    ap.add_argument("--budget", type=int, default=8192)
    ap.add_argument("--steps", type=int, default=300)
    a = ap.parse_args(argv)
    gc.collect()
    gc.freeze()        # as the service does at start-up
    res = run(a.requests, a.rows, a.prompt, a.output, a.budget, a.steps)
    print(json.dumps({"workload": vars(a), "host_ms": res}))
    return res


if __name__ == "__main__":
    main()
