"""Scheduler fuzzing without a model: random arrivals, prompt and output
lengths, stop tokens, cancellations, deadlines, prefix sharing and a tight KV
arena, with one or two plans in flight.  After every step the invariants
hold; every request reaches a terminal state within a bounded number of
steps (liveness) and every page returns to the free list or the prefix cache.
"""
import random

import pytest

from lunaflux_b200.config import CacheConfig, SchedulerConfig
from lunaflux_b200.contracts import SamplingParameters
from lunaflux_b200.prefix.radix import PrefixIdentity
from lunaflux_b200.scheduler.scheduler import AdmissionRejected, Request, Scheduler


def _run(seed: int, inflight: int, prefix: bool):
    rnd = random.Random(seed)
    now = [0.0]
    cfg = SchedulerConfig(step_token_budget=rnd.choice((16, 32, 64)), max_active_requests=rnd.choice((2, 4, 8)),
                          prefill_chunk_tokens=16, emergency_decode_page_reserve=1, waiting_age_threshold_steps=6)
    pages = rnd.randint(8, 24)
    s = Scheduler(cfg, CacheConfig(prefix_enabled=prefix), pages, PrefixIdentity("d" * 64, "", b"", 16, 2),
                  clock=lambda: now[0], max_context=200)
    s.max_inflight = inflight
    shared = [[rnd.randrange(100) for _ in range(32)] for _ in range(2)]
    rid = 0
    live = set()
    queued = []          # plans in flight, oldest first
    for step in range(3000):
        now[0] += 0.01
        if step < 300 and rnd.random() < 0.3:
            rid += 1
            n = rnd.randint(1, 60)
            prompt = (rnd.choice(shared) if rnd.random() < 0.4 else []) + [rnd.randrange(100) for _ in range(n)]
            req = Request(rid=rid, prompt=prompt[:150], max_new=rnd.randint(1, 30),
                          sampling=SamplingParameters(), stop_ids=frozenset({rnd.randrange(100)}),
                          deadline=now[0] + rnd.uniform(0.5, 5.0) if rnd.random() < 0.2 else None,
                          cache_scope=b"", cache_enabled=True, arrival=now[0])
            try:
                s.add_request(req)
                live.add(rid)
            except AdmissionRejected:
                pass
        if live and rnd.random() < 0.03:
            s.cancel(rnd.choice(sorted(live)))
        plan = s.schedule() if len(queued) < inflight else None
        if plan is not None:
            queued.append(plan)
        if queued and (len(queued) == inflight or plan is None):
            p = queued.pop(0)
            s.complete(p, [rnd.randrange(100) for r in p.rows if r.sample])
        for t in s.take_terminals():
            live.discard(t.rid)
        s.debug_check_invariants()
        if step >= 300 and not s.has_work() and not queued:
            break
    assert not live, f"requests never finished: {sorted(live)[:10]}"
    assert not s.has_work()
    held = s.prefix.page_count() if s.prefix is not None else 0
    assert s.allocator.allocated_page_count() == held


@pytest.mark.parametrize("seed", range(12))
@pytest.mark.parametrize("inflight", [1, 2])
def test_scheduler_fuzz(seed, inflight):
    _run(seed, inflight, prefix=seed % 2 == 0)
