"""Scheduler unit tests on deterministic fixtures: planning order, chunked
prefill, the emergency page reserve, admission, cancellation, deadlines,
completion validation, worker failure and rollback.

Modelled on the reference's scheduler/core tests (planning_test.mbt:
"build_next activates FIFO requests", "chunked prefill stays intermediate and
preserves decode reserve", "prefill may consume exactly to the emergency
reserve boundary", "decode is reserved first"; admission_token_bound_test.mbt;
completion_test.mbt: "stop token is published before terminal resource
release", "cancelled submitted work retires without post-cancel token";
registry_test.mbt: "waiting cancellation publishes slot-free notice and never
aliases re-admission", "deadline expiry is deterministic and leaves resource
owners balanced"; completion_wbtest.mbt: "device-state invalidation fails
active requests but preserves waiting work").  Every test ends with the
allocator and block tables balanced.
"""
import pytest

from lunaflux_b200.config import CacheConfig, SchedulerConfig
from lunaflux_b200.contracts import FinishReason, PublicErrorCode, RequestState, SamplingParameters
from lunaflux_b200.runtime.clock import FakeClock
from lunaflux_b200.scheduler.scheduler import AdmissionRejected, Request, Scheduler, SchedulerError

P = 16


def make(num_pages=64, budget=64, rows=8, chunk=64, reserve=0, age=64, waiting=64, max_context=512, clock=None):
    cfg = SchedulerConfig(step_token_budget=budget, max_active_requests=rows, max_waiting_requests=waiting,
                          prefill_chunk_tokens=chunk, emergency_decode_page_reserve=reserve,
                          waiting_age_threshold_steps=age, output_event_capacity=max(rows, budget))
    return Scheduler(cfg, CacheConfig(prefix_enabled=False), num_pages, clock=clock or FakeClock(),
                     max_context=max_context)


def req(rid, n=10, max_new=4, stop=(), deadline=None, first=100):
    return Request(rid, list(range(first, first + n)), max_new, SamplingParameters(), frozenset(stop),
                   deadline=deadline)


def run_step(s, tokens=None):
    """Plans one step and completes it with ``tokens`` (default 7 per sampling row)."""
    plan = s.schedule()
    assert plan is not None
    n = len(plan.sample_rows)
    outs = s.complete(plan, tokens if tokens is not None else [7] * n)
    s.debug_check_invariants()
    return plan, outs


def balanced(s):
    s.debug_check_invariants()
    assert not s.running and not s.waiting and not s.inflight
    assert s.allocator.free_page_count() == s.allocator.capacity
    assert s.tables.free_table_count() == s.cfg.max_active_requests


# ----------------------------------------------------------------------------- planning
def test_fifo_activation_then_decode_rows_in_running_order():
    s = make()
    for rid in (3, 1, 2):
        s.add_request(req(rid, n=5 + rid))
    plan, outs = run_step(s)
    assert [r.req.rid for r in plan.rows] == [3, 1, 2]
    assert all(not r.decode and r.sample and r.start == 0 for r in plan.rows)
    assert [r.n for r in plan.rows] == [8, 6, 7]
    assert [o.rid for o in outs] == [3, 1, 2] and all(o.token == 7 for o in outs)
    assert [o.position for o in outs] == [8, 6, 7]
    plan, _ = run_step(s)
    assert [r.req.rid for r in plan.rows] == [3, 1, 2]
    assert all(r.decode and r.n == 1 for r in plan.rows)
    assert [r.start for r in plan.rows] == [8, 6, 7]   # the first sampled token's position


def test_idle_scheduler_plans_nothing_and_one_plan_in_flight_at_a_time():
    s = make()
    assert s.schedule() is None and not s.has_work()
    s.add_request(req(1))
    plan = s.schedule()
    with pytest.raises(SchedulerError):
        s.schedule()
    s.complete(plan, [5])
    assert s.schedule() is not None


def test_decode_rows_are_reserved_before_prefill_and_serialised_after_it():
    s = make(budget=4, chunk=4)
    s.add_request(req(1, n=3))
    s.add_request(req(2, n=3))
    while any(r.state is RequestState.PREFILL or r.state is RequestState.WAITING for r in s.requests.values()):
        run_step(s)
    s.add_request(req(3, n=20))
    plan = s.schedule()
    kinds = [(r.req.rid, r.decode) for r in plan.rows]
    # two decode rows got their tokens first; the prefill takes what is left
    assert kinds == [(3, False), (1, True), (2, True)]
    assert plan.rows[0].n == 2 and not plan.rows[0].sample
    s.complete(plan, [9, 9])


def test_chunked_prefill_stays_intermediate_until_its_last_chunk():
    s = make(budget=16, chunk=16)
    s.add_request(req(1, n=40))
    seen = []
    for _ in range(3):
        plan, outs = run_step(s)
        (row,) = plan.rows
        seen.append((row.start, row.n, row.sample))
        r = s.requests[1]
        if row.sample:
            assert r.state is RequestState.DECODE and [o.token for o in outs] == [7]
        else:
            assert r.state is RequestState.PREFILL and outs == []
    assert seen == [(0, 16, False), (16, 16, False), (32, 8, True)]
    assert s.requests[1].num_computed == 40 and len(s.requests[1].pages) == 3


def test_new_admission_leaves_the_emergency_reserve_untouched():
    # 10 pages, reserve 4: a running decode keeps the reserve for itself
    s = make(num_pages=10, budget=256, chunk=256, reserve=4)
    s.add_request(req(1, n=P - 1, max_new=40))
    run_step(s)                                   # rid 1 holds 1 page; its next decode fits in it
    assert s.allocator.free_page_count() == 9
    s.add_request(req(2, n=5 * P))                # needs 5 pages: 9 - 5 = 4 == reserve, admitted
    plan, _ = run_step(s)
    assert [(r.req.rid, r.decode) for r in plan.rows] == [(2, False), (1, True)]
    assert s.allocator.free_page_count() == 4
    s.add_request(req(3, n=P))                    # one more page would dip into the reserve
    plan, _ = run_step(s)
    assert 3 not in {r.req.rid for r in plan.rows}
    assert s.requests[3].state is RequestState.WAITING


def test_first_admission_may_use_the_reserve_when_nothing_runs():
    s = make(num_pages=6, budget=256, chunk=256, reserve=4)
    s.add_request(req(1, n=5 * P - 1))
    plan, _ = run_step(s)
    assert plan.rows[0].req.rid == 1 and s.allocator.free_page_count() == 1


def test_aged_waiting_request_goes_before_partial_prefills():
    s = make(budget=8, chunk=8, age=2, rows=4)
    s.add_request(req(1, n=64))                   # long prefill, 8 tokens per step
    run_step(s)
    s.add_request(req(2, n=4))
    plan, _ = run_step(s)
    assert [r.req.rid for r in plan.rows] == [1]  # partial prefill first while rid 2 is young
    run_step(s)
    plan, _ = run_step(s)                          # rid 2 waited 2 steps: aged, admitted first
    assert plan.rows[0].req.rid == 2


# ----------------------------------------------------------------------------- admission
def test_admission_rejections_mutate_nothing():
    s = make(num_pages=4, waiting=2, max_context=128)
    s.add_request(req(1))
    gen, waiting = s.generation, list(s.waiting)
    cases = [
        (req(1), PublicErrorCode.INVALID_REQUEST),                # duplicate live id
        (req(9, n=0), PublicErrorCode.CONTEXT_OVERFLOW),          # empty prompt
        (req(9, n=128), PublicErrorCode.CONTEXT_OVERFLOW),        # prompt fills the whole context
        (req(9, n=4 * P), PublicErrorCode.CONTEXT_OVERFLOW),      # prompt + one page beyond the arena
    ]
    for r, code in cases:
        with pytest.raises(AdmissionRejected) as e:
            s.add_request(r)
        assert e.value.code is code
        assert s.generation == gen and list(s.waiting) == waiting and set(s.requests) == {1}
    s.add_request(req(2))
    with pytest.raises(AdmissionRejected) as e:
        s.add_request(req(3))
    assert e.value.code is PublicErrorCode.OVERLOADED and set(s.requests) == {1, 2}


def test_prompt_bound_is_the_tightest_ceiling():
    s = make(max_context=64)
    r = req(1, n=10)
    r.context_ceiling = 20
    s.add_request(r)
    assert r.context_ceiling == 20
    r2 = req(2, n=10)
    s.add_request(r2)
    assert r2.context_ceiling == 64
    with pytest.raises(AdmissionRejected):
        s.add_request(req(3, n=64))


# ----------------------------------------------------------------------------- lifecycle
def test_waiting_cancellation_publishes_one_terminal_and_the_id_is_reusable():
    s = make()
    s.add_request(req(1))
    g = s.requests[1].generation
    assert s.cancel(1) is True
    assert s.cancel(1) is False and s.cancel(99) is False
    (t,) = s.take_terminals()
    assert (t.rid, t.reason, t.error) == (1, FinishReason.CANCELLED, None)
    assert s.take_terminals() == []
    s.add_request(req(1))
    assert s.requests[1].generation > g
    run_step(s)
    assert s.take_terminals() == []


def test_cancelled_in_flight_work_retires_without_a_token():
    s = make()
    s.add_request(req(1))
    s.add_request(req(2))
    plan = s.schedule()
    assert s.cancel(1)
    assert s.allocator.free_page_count() == s.allocator.capacity - 1   # rid 1's page is back already
    outs = s.complete(plan, [5, 6])
    assert [(o.rid, o.token) for o in outs] == [(2, 6)]
    s.cancel(2)
    s.take_terminals()
    balanced(s)


def test_stop_token_is_published_with_the_terminal_and_resources_released():
    s = make()
    s.add_request(req(1, stop=(42,), max_new=10))
    run_step(s)
    _, outs = run_step(s, [42])
    (o,) = outs
    assert (o.token, o.finished, o.reason) == (42, True, FinishReason.STOP_SEQUENCE)
    (t,) = s.take_terminals()
    assert t.reason is FinishReason.STOP_SEQUENCE and t.error is None
    balanced(s)


@pytest.mark.parametrize("ceiling", [None, 13])
def test_token_limit_and_context_ceiling_finish_with_token_limit(ceiling):
    s = make()
    r = req(1, n=10, max_new=5)
    if ceiling:
        r.context_ceiling = ceiling
    s.add_request(r)
    toks = []
    while s.has_work():
        _, outs = run_step(s)
        toks += outs
    want = 5 if ceiling is None else ceiling - 10
    assert len(toks) == want and toks[-1].finished and toks[-1].reason is FinishReason.TOKEN_LIMIT
    assert not any(o.finished for o in toks[:-1])
    assert [o.position for o in toks] == list(range(10, 10 + want))
    balanced(s)


def test_deadline_expiry_is_deterministic_and_balances_resources():
    clock = FakeClock()
    s = make(clock=clock)
    s.add_request(req(1, deadline=clock() + 1.0))
    s.add_request(req(2, deadline=clock() + 5.0))
    s.add_request(req(3, deadline=clock() + 1.0))
    run_step(s)
    clock.advance(1.0)                            # exactly at the deadline: expired
    plan = s.schedule()
    assert [r.req.rid for r in plan.rows] == [2]
    ts = s.take_terminals()
    assert [(t.rid, t.error) for t in ts] == [(1, PublicErrorCode.DEADLINE_EXCEEDED),
                                                (3, PublicErrorCode.DEADLINE_EXCEEDED)]
    s.complete(plan, [1])
    clock.advance(0.5)
    run_step(s)
    assert s.take_terminals() == [] and 2 in s.requests
    s.cancel(2)
    balanced(s)


def test_worker_failure_fails_active_requests_and_keeps_waiting_ones():
    s = make(rows=2)
    for rid in (1, 2, 3):
        s.add_request(req(rid))
    plan = s.schedule()
    assert {r.req.rid for r in plan.rows} == {1, 2}
    s.abort_plan(plan)
    s.fail_active()
    ts = s.take_terminals()
    assert [(t.rid, t.error) for t in ts] == [(1, PublicErrorCode.WORKER_UNAVAILABLE),
                                                (2, PublicErrorCode.WORKER_UNAVAILABLE)]
    assert list(s.requests) == [3] and s.requests[3].state is RequestState.WAITING
    assert s.allocator.free_page_count() == s.allocator.capacity
    _, outs = run_step(s)
    assert [o.rid for o in outs] == [3]


# ----------------------------------------------------------------------------- completion
def test_completion_is_validated_before_anything_moves():
    s = make()
    s.add_request(req(1))
    s.add_request(req(2))
    plan = s.schedule()
    with pytest.raises(SchedulerError):
        s.complete(plan, [1])                     # one token for two sampling rows
    with pytest.raises(SchedulerError):
        s.complete(plan, [1, 2, 3])
    assert s.inflight == [plan] and all(r.output == [] for r in s.requests.values())
    other = type(plan)(plan.seq + 100, [])
    with pytest.raises(SchedulerError):
        s.complete(other, [])                     # not the oldest plan in flight
    outs = s.complete(plan, [1, 2])               # the exact retry still commits
    assert [(o.rid, o.token) for o in outs] == [(1, 1), (2, 2)]


def test_overlapped_plans_complete_in_plan_order():
    s = make()
    s.max_inflight = 2
    s.add_request(req(1, max_new=8))
    p1 = s.schedule()
    p2 = s.schedule()
    assert p2.rows[0].decode and p2.rows[0].fwd == 0     # reads p1's sample on the device
    with pytest.raises(SchedulerError):
        s.complete(p2, [2])
    s.complete(p1, [1])
    s.complete(p2, [2])
    assert s.requests[1].output == [1, 2]


def test_abort_plan_drops_it_and_every_later_plan():
    s = make()
    s.max_inflight = 2
    s.add_request(req(1, max_new=8))
    p1 = s.schedule()
    s.schedule()
    s.abort_plan(p1)
    assert s.inflight == []


# ----------------------------------------------------------------------------- pressure
def test_preemption_recomputes_the_youngest_and_keeps_the_oldest_growing():
    # 6 pages: two requests of 2 pages each grow until one must give way
    s = make(num_pages=6, budget=256, chunk=256, rows=4)
    s.add_request(req(1, n=2 * P, max_new=40, first=10))
    s.add_request(req(2, n=2 * P, max_new=40, first=500))
    outs_by = {1: [], 2: []}
    steps = 0
    while s.has_work() and steps < 200:
        _, outs = run_step(s)
        for o in outs:
            outs_by[o.rid].append(o)
        steps += 1
    assert s.preemptions >= 1
    assert len(outs_by[1]) == 40 and len(outs_by[2]) == 40
    # positions are contiguous per request even across the recompute
    for rid in (1, 2):
        assert [o.position for o in outs_by[rid]] == list(range(2 * P, 2 * P + 40))
    balanced(s)


def test_a_request_that_cannot_fit_alone_fails_with_context_overflow():
    s = make(num_pages=3, budget=256, chunk=256, max_context=512)
    s.add_request(req(1, n=2 * P - 1, max_new=100))    # admitted: 2 pages + 1 to grow
    for _ in range(60):
        if not s.has_work():
            break
        plan = s.schedule()
        if plan is None:
            break
        s.complete(plan, [7] * len(plan.sample_rows))
    (t,) = s.take_terminals()
    assert t.rid == 1 and t.error is PublicErrorCode.CONTEXT_OVERFLOW
    balanced(s)
