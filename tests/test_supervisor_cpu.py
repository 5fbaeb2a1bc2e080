"""Supervised rank processes on CPU (gloo): lock-step serving, and recovery
from a rank that dies, stops answering, or whose device fails.  Failures are
made on the host: a rank process exits, stops itself (SIGSTOP) so its
heartbeats cease, or runs on the fake device whose kernel launch raises."""
import os
import signal

import pytest
import torch

from lunaflux_b200.contracts import PublicErrorCode
from lunaflux_b200.engine.supervisor import Supervisor


def _spec():
    from lunaflux_b200.models.spec import LlamaSpec
    return LlamaSpec(hidden=64, layers=2, heads=4, kv_heads=2, head_dim=16, ffn=172, vocab=256, max_position=512,
                     dtype="fp32")


class _FaultyEngine:
    """Wraps an engine; on the configured rank / generation / step it fails."""

    def __init__(self, eng, rank):
        self.eng = eng
        self.rank = rank
        self.steps = 0
        self.mode = os.environ.get("LF_TEST_FAULT", "")
        self.gen = int(os.environ.get("LUNAFLUX_GENERATION", "1"))

    def __getattr__(self, k):
        return getattr(self.eng, k)

    def step(self):
        self.steps += 1
        if self.rank == 1 and self.gen == 1 and self.steps == 3:
            if self.mode == "exit":
                os._exit(3)
            if self.mode == "stop":
                os.kill(os.getpid(), signal.SIGSTOP)
        return self.eng.step()


def tiny_factory(rank, world):
    import torch.distributed as dist

    from lunaflux_b200.config import CacheConfig, SchedulerConfig
    from lunaflux_b200.engine.engine import EngineOptions, LLMEngine
    from lunaflux_b200.models.weights import build_runtime, random_checkpoint
    from lunaflux_b200.ops.torch_ops import TorchOps
    from lunaflux_b200.parallel.comm import TPComm
    from lunaflux_b200.parallel.tp import TPShard
    import datetime
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=30))
    spec = _spec()
    ck = random_checkpoint(spec, 0)
    w = build_runtime(spec, lambda n: ck[n], TPShard(rank, world, spec))
    ops = TorchOps()
    if os.environ.get("LF_TEST_FAULT") == "device" and rank == 1 and os.environ.get("LUNAFLUX_GENERATION") == "1":
        # a kernel launch that fails on the fake device in the third forward
        from lunaflux_b200.testing import FakeDeviceOps, FaultPlan
        ops = FakeDeviceOps(FaultPlan(at_forward=3, kind="launch_error"))
    eng = LLMEngine(w, ops, "cpu", SchedulerConfig(step_token_budget=64, max_active_requests=4,
                                                          prefill_chunk_tokens=64, emergency_decode_page_reserve=1),
                    CacheConfig(), EngineOptions(max_context=256, num_pages=64, graph_sizes=()), comm=TPComm())
    return _FaultyEngine(eng, rank)


def _expect(prompts, n):
    from lunaflux_b200.models.weights import random_checkpoint
    from lunaflux_b200.oracle.reference import ReferenceModel
    ref = ReferenceModel(_spec(), random_checkpoint(_spec(), 0))
    return [ref.generate_greedy(p, n) for p in prompts]


PROMPTS = [[5, 6, 7], [9, 10, 11, 12, 13], [1, 2, 3, 4], [200, 100]]


@pytest.mark.parametrize("fault", ["", "exit", "stop", "device"])
def test_supervised_tp_ranks(fault, monkeypatch):
    monkeypatch.setenv("LF_TEST_FAULT", fault)
    sup = Supervisor(2, tiny_factory, heartbeat_s=0.1, dead_after_s=2.0, step_timeout_s=60.0)
    sup.start()
    try:
        sup.submit(1, PROMPTS[0], 6)
        sup.submit(2, PROMPTS[1], 6)
        sup.step()
        sup.step()
        sup.submit(3, PROMPTS[2], 6)
        sup.submit(4, PROMPTS[3], 6)
        sup.run_until_done()
    finally:
        sup.close()
    expect = _expect(PROMPTS, 6)
    if not fault:
        assert sup.failures == 0
        for i in range(4):
            assert sup.reqs[i + 1].tokens == expect[i]
        return
    assert sup.failures == 1 and sup.generation == 2
    # requests that were producing tokens fail retryably; the ones still
    # waiting survive and complete correctly in the new generation
    for rid in (1, 2):
        assert sup.reqs[rid].error is PublicErrorCode.WORKER_UNAVAILABLE
    for rid in (3, 4):
        assert sup.reqs[rid].error is None and sup.reqs[rid].tokens == expect[rid - 1]


def test_service_over_supervised_ranks_survives_a_lost_rank(monkeypatch):
    """The serving path on supervised rank processes: rank 1 exits in its
    third step.  The service keeps running; the requests that were producing
    tokens fail with the retryable worker_unavailable code, the ones still
    waiting complete in the next generation with the oracle's tokens, and a
    request submitted after the recovery completes too."""
    import threading
    import time

    from lunaflux_b200.contracts import GenerateRequest
    from lunaflux_b200.engine.engine import EngineOptions
    from lunaflux_b200.engine.supervised import SupervisedEngine
    from lunaflux_b200.contracts import CompletedEvent, FailedEvent, TokenEvent
    from lunaflux_b200.service.server import EngineService
    from lunaflux_b200.contracts import default_limits

    monkeypatch.setenv("LF_TEST_FAULT", "exit")
    sup = Supervisor(2, tiny_factory, heartbeat_s=0.1, dead_after_s=2.0, step_timeout_s=60.0)
    sup.start()
    eng = SupervisedEngine(sup, _spec(), EngineOptions(max_context=256), time.monotonic)
    svc = EngineService(eng, None, default_limits(256, 256))
    events = {}
    done = {}
    lock = threading.Lock()

    def sink_for(rid):
        def sink(ev):
            with lock:
                events.setdefault(rid, []).append(ev)
                if isinstance(ev, (CompletedEvent, FailedEvent)):
                    done[rid] = ev
        return sink

    def wait_for(rids, timeout=120.0):
        t0 = time.monotonic()
        while time.monotonic() - t0 < timeout:
            with lock:
                if all(r in done for r in rids):
                    return
            time.sleep(0.02)
        raise AssertionError(f"requests {rids} did not finish: {sorted(done)}")

    svc.start()
    try:
        for rid in (1, 2):
            svc.submit(GenerateRequest(request_id=rid, input_tokens=tuple(PROMPTS[rid - 1]), max_new_tokens=6),
                       sink_for(rid))
        # the first two produce tokens before the fault; the next two wait until then
        t0 = time.monotonic()
        while time.monotonic() - t0 < 60:
            with lock:
                if all(any(isinstance(e, TokenEvent) for e in events.get(r, [])) for r in (1, 2)):
                    break
            time.sleep(0.01)
        for rid in (3, 4):
            svc.submit(GenerateRequest(request_id=rid, input_tokens=tuple(PROMPTS[rid - 1]), max_new_tokens=6),
                       sink_for(rid))
        wait_for([1, 2, 3, 4])
        svc.submit(GenerateRequest(request_id=5, input_tokens=tuple(PROMPTS[0]), max_new_tokens=6), sink_for(5))
        wait_for([5])
        assert svc.alive()
    finally:
        svc.stop()
        eng.close()
    expect = _expect(PROMPTS, 6)
    assert sup.failures == 1 and sup.generation == 2
    for rid in (1, 2):
        ev = done[rid]
        assert isinstance(ev, FailedEvent) and ev.code is PublicErrorCode.WORKER_UNAVAILABLE and ev.retryable, ev
    for rid, want in ((3, expect[2]), (4, expect[3]), (5, expect[0])):
        assert isinstance(done[rid], CompletedEvent), done[rid]
        toks = [e.token_id for e in events[rid] if isinstance(e, TokenEvent)]
        assert toks == want, (rid, toks, want)
        # positions count from the prompt, as the in-process engine reports them
        n = len(PROMPTS[(rid - 1) % 4])
        assert [e.position for e in events[rid] if isinstance(e, TokenEvent)] == list(range(n, n + 6))


def failing_factory(rank, world):
    if rank == 1:
        raise RuntimeError("model directory unreadable")
    import time
    time.sleep(0.5)
    return tiny_factory(rank, world)


def test_a_rank_that_cannot_start_fails_the_start_and_leaves_nothing_running():
    """Startup handshake (reference: worker_process 'startup handshake rejects
    an incompatible child before readiness'): a rank whose engine cannot be
    built reports the error; start() raises and every rank of that
    generation is reaped."""
    from lunaflux_b200.engine.supervisor import WorkerLost
    sup = Supervisor(2, failing_factory, heartbeat_s=0.1, dead_after_s=2.0, step_timeout_s=60.0)
    with pytest.raises(WorkerLost, match="rank 1"):
        sup.start()
    assert sup.procs == [] and sup.conns == []


def test_cancel_and_close_through_the_supervisor(monkeypatch):
    """A request cancelled between steps ends CANCELLED on every rank while
    the other completes with the oracle's tokens; close() reaps every rank."""
    monkeypatch.setenv("LF_TEST_FAULT", "")
    sup = Supervisor(2, tiny_factory, heartbeat_s=0.1, dead_after_s=2.0, step_timeout_s=60.0)
    sup.start()
    procs = list(sup.procs)
    try:
        sup.submit(1, PROMPTS[0], 40)
        sup.submit(2, PROMPTS[1], 6)
        sup.step()
        sup.step()
        sup.cancel(1)
        sup.run_until_done()
    finally:
        sup.close()
    assert all(not p.is_alive() for p in procs)
    assert sup.reqs[1].done and sup.reqs[1].reason == "CANCELLED" and len(sup.reqs[1].tokens) < 40
    assert sup.reqs[2].tokens == _expect([PROMPTS[1]], 6)[0] and sup.reqs[2].reason == "TOKEN_LIMIT"
    assert sup.failures == 0
