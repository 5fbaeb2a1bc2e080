"""The serving engine over supervised rank processes.

``SupervisedEngine`` gives ``service.server.EngineService`` the engine
interface it drives (submit / cancel / step / has_work, token listeners,
terminal results, scheduler.cancel / fail_active, metrics) on top of
``engine.supervisor.Supervisor``: every tensor-parallel rank is a child
process with its own GPU and engine shard, and the front process that serves
TCP / HTTP holds no GPU state.  A rank that exits, raises, stops answering
heartbeats or fails a step ends its generation: requests that were producing
tokens fail with the retryable ``worker_unavailable`` code, requests that had
not started are re-submitted to the next generation, and the service keeps
running.

Reference: engine/worker_service/README.mbt.md:93-104 (worker failure fails
the device-backed requests and keeps the waiting ones) and
engine/worker_process/README.mbt.md:70-80 (ordered recovery, generations).
"""
from __future__ import annotations

from typing import Callable, Dict, List, Optional

from ..contracts import FinishReason, PublicErrorCode
from ..metrics import EngineMetrics
from ..scheduler.scheduler import TokenOutput
from .engine import RequestResult
from .supervisor import Supervisor, WorkerLost


class _SchedulerView:
    def __init__(self, eng: "SupervisedEngine"):
        self._eng = eng

    def cancel(self, rid: int) -> bool:
        return self._eng.cancel(rid)

    def fail_active(self, code: PublicErrorCode):
        for rid, st in list(self._eng._live.items()):
            if st["tokens"]:
                self._eng._terminal(rid, None, code)


class SupervisedEngine:
    def __init__(self, supervisor: Supervisor, spec, opts, clock: Callable[[], float]):
        self.sup = supervisor
        self.spec = spec
        self.opts = opts
        self.clock = clock
        self.listeners: List[Callable] = []
        self.results: Dict[int, RequestResult] = {}
        self.metrics = EngineMetrics()
        self.scheduler = _SchedulerView(self)
        self._live: Dict[int, dict] = {}
        self._next_rid = 1

    @property
    def failures(self) -> int:
        return self.sup.failures

    # ------------------------------------------------------------ requests
    def add_request(self, prompt, max_new_tokens: int, sampling=None, stop_ids=(), rid: Optional[int] = None,
                    deadline_s=None, cache_scope=b"", use_prefix_cache=True, arrival=None) -> int:
        from .engine import check_token_ids
        prompt = list(prompt)
        check_token_ids(prompt, self.spec.vocab)     # rejected here, before any rank sees it
        if rid is None:
            rid = self._next_rid
        self._next_rid = max(self._next_rid, rid + 1)
        self.sup.submit(rid, prompt, max_new_tokens, sampling, tuple(stop_ids))
        now = self.clock()
        self._live[rid] = {"prompt_len": len(prompt), "tokens": [], "arrival": now if arrival is None
                           else arrival, "first": None,
                           "deadline": None if deadline_s is None else now + deadline_s}
        return rid

    def submit(self, g) -> int:
        if g.input_tokens is None:
            raise ValueError("text requests must be tokenized by the service layer first")
        return self.add_request(g.input_tokens, g.max_new_tokens, g.sampling, g.stop.token_ids, rid=g.request_id,
                                deadline_s=None if g.deadline_millis is None else g.deadline_millis / 1000.0)

    def cancel(self, rid: int) -> bool:
        if rid not in self._live:
            return False
        self._cancel_on_ranks(rid)
        return True

    def _cancel_on_ranks(self, rid: int):
        # a rank lost here is found again, and recovered from, by the next step
        try:
            self.sup.cancel(rid)
        except WorkerLost:
            pass

    def has_work(self) -> bool:
        return bool(self._live)

    # ------------------------------------------------------------ steps
    def _terminal(self, rid: int, reason: Optional[FinishReason], error: Optional[PublicErrorCode]):
        st = self._live.pop(rid, None)
        self.sup.reqs.pop(rid, None)      # the supervisor keeps only requests still in flight
        if st is None:
            return
        self.results[rid] = RequestResult(rid, st["prompt_len"], st["tokens"], reason, error, st["arrival"],
                                          st["first"], self.clock(), 0)
        if error is not None:
            self.metrics.failed.inc(code=error.name.lower())
        else:
            self.metrics.finished.inc(reason=reason.name.lower() if reason else "none")

    def _expire_deadlines(self):
        # the ranks' schedulers are not told deadlines: they expire here, in
        # the front process, and the ranks get a cancel
        now = self.clock()
        for rid, st in list(self._live.items()):
            if st["deadline"] is not None and now >= st["deadline"]:
                self._terminal(rid, None, PublicErrorCode.DEADLINE_EXCEEDED)
                self._cancel_on_ranks(rid)

    def step(self) -> List[TokenOutput]:
        self._expire_deadlines()
        failures = self.sup.failures
        self.sup.step()
        outs: List[TokenOutput] = []
        if self.sup.failures != failures:
            # a rank was lost: the recovery failed the requests that had produced tokens
            for rid in self.sup.last_failed:
                self._terminal(rid, None, PublicErrorCode.WORKER_UNAVAILABLE)
            return outs
        done = {rid: (reason, error) for rid, reason, error in self.sup.last_done}
        now = self.clock()
        for rid, token, finished in self.sup.last_outs:
            st = self._live.get(rid)
            if st is None:
                continue
            if st["first"] is None:
                st["first"] = now
            st["tokens"].append(token)
            reason = None
            if finished:
                r = done.get(rid, (None, None))[0]
                reason = FinishReason[r] if r else FinishReason.TOKEN_LIMIT
            # position in the sequence, as the in-process engine reports it
            outs.append(TokenOutput(rid, token, st["prompt_len"] + len(st["tokens"]) - 1, finished, reason))
        if outs:
            self.metrics.output_tokens.inc(len(outs))
            for cb in self.listeners:
                cb(outs)
        for rid, (reason, error) in done.items():
            self._terminal(rid, FinishReason[reason] if reason else None, PublicErrorCode[error] if error else None)
        return outs

    def _drain_terminals(self):
        pass

    def close(self):
        self.sup.close()
