"""Planning cost does not grow with the waiting queue.

A step plans over the running rows and admits from the head of the queue;
with thousands of requests queued (a Poisson burst, configuration #5) its
cost must stay flat.  The check counts the time of ``schedule`` for the same
256-row decode state with 64 and with 4096 waiting requests, after every one
of them has aged past the starvation threshold (the case that used to be
quadratic in the queue length)."""
import time

from lunaflux_b200.config import CacheConfig, SchedulerConfig
from lunaflux_b200.contracts import SamplingParameters
from lunaflux_b200.scheduler.scheduler import Request, Scheduler


def _plan_ms(queued: int) -> float:
    rows = 256
    cfg = SchedulerConfig(step_token_budget=rows, max_active_requests=rows, prefill_chunk_tokens=rows,
                          emergency_decode_page_reserve=8, waiting_age_threshold_steps=4,
                          max_waiting_requests=rows + queued)
    s = Scheduler(cfg, CacheConfig(prefix_enabled=False), rows * 8 + 64, None, max_context=512)
    for i in range(rows + queued):
        s.add_request(Request(rid=i + 1, prompt=[1 + i % 7] * 8, max_new=400, sampling=SamplingParameters()))
    times = []
    for step in range(40):
        t0 = time.perf_counter()
        plan = s.schedule()
        times.append(time.perf_counter() - t0)
        s.complete(plan, [5] * len(plan.sample_rows))
    assert len(s.running) == rows and len(s.waiting) == queued
    times.sort()
    return times[len(times) // 2] * 1e3


def test_planning_cost_is_flat_in_the_queue_length():
    small = min(_plan_ms(64) for _ in range(2))
    large = min(_plan_ms(4096) for _ in range(2))
    assert large < 3.0 * small + 0.5, f"{large:.2f} ms with 4096 queued vs {small:.2f} ms with 64"


def test_completion_validates_before_mutation():
    """A completion must carry exactly one token per sampling row and be for
    the oldest plan in flight; a rejected one changes nothing and the correct
    completion still applies (reference: engine/worker_protocol completion
    validation rejects wrong counts and stale plans without mutation)."""
    import pytest
    from lunaflux_b200.scheduler.scheduler import SchedulerError
    cfg = SchedulerConfig(step_token_budget=64, max_active_requests=4, prefill_chunk_tokens=8,
                          emergency_decode_page_reserve=1)
    s = Scheduler(cfg, CacheConfig(prefix_enabled=False), 32, None, max_context=128)
    s.max_inflight = 2
    for i in range(3):
        s.add_request(Request(rid=i + 1, prompt=[1 + i] * 12, max_new=3, sampling=SamplingParameters()))
    first = s.schedule()           # chunks of 8: no row finishes its prompt, nothing sampled
    second = s.schedule()          # the remaining 4 tokens: every row samples
    assert not first.sample_rows and len(second.sample_rows) == 3
    before = [(r.num_computed, list(r.output), r.pending) for r in s.running]
    with pytest.raises(SchedulerError):
        s.complete(second, [5, 5, 5])          # not the oldest in flight
    with pytest.raises(SchedulerError):
        s.complete(first, [5])                 # a token for a row that samples nothing
    assert [(r.num_computed, list(r.output), r.pending) for r in s.running] == before
    assert s.inflight == [first, second]
    s.complete(first, [])
    with pytest.raises(SchedulerError):
        s.complete(second, [5, 5])             # one token short
    outs = s.complete(second, [5, 6, 7])
    assert [o.token for o in outs] == [5, 6, 7] and not s.inflight


def test_host_step_benchmark_runs_small():
    from lunaflux_b200.bench.host import run
    res = run(requests=64, rows=16, prompt=96, output=8, budget=256, steps=80)
    assert res["prefill"]["steps"] > 0 and res["decode"]["steps"] > 0
    assert all(v >= 0 for kind in res.values() for v in kind.values())
