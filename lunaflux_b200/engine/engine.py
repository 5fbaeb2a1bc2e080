"""The engine core: scheduler + model runner in one loop.

``LLMEngine`` is the single-process, single-rank engine (TP = 1) and the
rank-0 driver of a tensor-parallel group.  Its busy loop is
schedule -> execute (one packed upload, one graph replay or eager forward,
on-device sampling, one int32 readback) -> complete (scheduler commit,
events).  Reference: engine/worker_service (WorkerService::progress,
progress.mbt:121) joined with engine/device_worker (execute_frame,
execute.mbt:41-70); here both run in one process per GPU with no socket in
the data path.
"""
from __future__ import annotations

import dataclasses
import time
from typing import Callable, Dict, Iterable, List, Optional, Sequence, Union

import numpy as np
import torch

from ..config import CacheConfig, SchedulerConfig
from ..contracts import (CompletedEvent, FailedEvent, FinishReason, GenerateRequest, PublicErrorCode,
                         SamplingParameters, TokenEvent, Usage)
from ..kv.layout import kv_bytes_per_page
from ..metrics import EngineMetrics
from ..models.spec import LlamaSpec
from ..models.weights import ModelWeights
from ..prefix.radix import PrefixIdentity
from ..scheduler.scheduler import AdmissionRejected, Request, Scheduler, StepPlan, TokenOutput
from .runner import ModelRunner, StepFailed  # noqa: F401  (re-exported)


@dataclasses.dataclass
class EngineOptions:
    max_context: int = 4096
    num_pages: int = 0                     # 0: derive from free memory
    memory_fraction: float = 0.90          # of free device memory after weights, for the KV arena
    graph_sizes: Sequence[int] = (1, 2, 4, 8, 16, 24, 32, 48, 64, 96, 128, 160, 192, 224, 256)
    check_errors_every: int = 16
    tokenizer_digest: str = ""
    sequence_parallel: bool = False        # TP only: residual stream sharded by tokens (reduce-scatter / all-gather)
    overlap_steps: bool = False            # plan and launch step n+1 before step n's tokens reach the host
    tp_sample_candidates: bool = False     # TP stochastic sampling from per-shard top-k candidates (top_k <= 64)
    moe_all_to_all: bool = False           # with sequence parallelism: experts by dispatch / combine all-to-all


@dataclasses.dataclass
class RequestResult:
    rid: int
    prompt_len: int
    tokens: List[int]
    reason: Optional[FinishReason]
    error: Optional[PublicErrorCode]
    arrival: float
    first_token_time: Optional[float]
    finish_time: Optional[float]
    cached_tokens: int

    @property
    def ttft(self) -> Optional[float]:
        return None if self.first_token_time is None else self.first_token_time - self.arrival

    @property
    def tpot(self) -> Optional[float]:
        if self.first_token_time is None or self.finish_time is None or len(self.tokens) < 2:
            return None
        return (self.finish_time - self.first_token_time) / (len(self.tokens) - 1)


def check_token_ids(toks, vocab: int):
    """Admission rejects prompt ids outside the loaded vocabulary (they would
    otherwise reach the embedding kernel and fail the whole step)."""
    if toks and (min(toks) < 0 or max(toks) >= vocab):
        raise AdmissionRejected(PublicErrorCode.INVALID_REQUEST, "prompt token id outside the model's vocabulary")


class LLMEngine:
    def __init__(self, weights: ModelWeights, ops, device, sched: SchedulerConfig = SchedulerConfig(),
                 cache: CacheConfig = CacheConfig(), opts: EngineOptions = EngineOptions(), comm=None,
                 clock: Callable[[], float] = time.monotonic):
        self.spec: LlamaSpec = weights.spec
        self.device = torch.device(device)
        self.opts = opts
        self.clock = clock
        P = cache.tokens_per_page
        num_pages = opts.num_pages or self._pages_from_memory(weights, cache, sched, opts)
        ident = PrefixIdentity(self.spec.paged_plan_digest(P, cache.layout_version), opts.tokenizer_digest, b"", P,
                               cache.layout_version)
        self.scheduler = Scheduler(sched, cache, num_pages, ident, clock=clock, max_context=opts.max_context)
        self.runner = ModelRunner(weights, ops, device, num_pages, sched.step_token_budget + sched.max_rows_per_step,
                                  sched.max_rows_per_step, opts.max_context, P, opts.graph_sizes, comm=comm,
                                  check_errors_every=opts.check_errors_every,
                                  sequence_parallel=opts.sequence_parallel, overlap=opts.overlap_steps,
                                  sample_candidates=opts.tp_sample_candidates, moe_all_to_all=opts.moe_all_to_all)
        if opts.overlap_steps:
            self.scheduler.max_inflight = 2
        self._launched: List[tuple] = []       # (plan, runner handle, t0), oldest first
        self.results: Dict[int, RequestResult] = {}
        self.live: Dict[int, Request] = {}
        self._next_rid = 1
        self.listeners: List[Callable] = []
        self.metrics = EngineMetrics()

    def _pages_from_memory(self, weights, cache, sched, opts) -> int:
        per_page = kv_bytes_per_page(self.spec, weights.shard.kv_heads, cache.tokens_per_page,
                                     weights.embed.element_size())
        want = sched.max_active_requests * -(-opts.max_context // cache.tokens_per_page) + 64
        if self.device.type != "cuda":
            return want
        free, _ = torch.cuda.mem_get_info(self.device)
        reserve = 6 << 30  # activations, logits, graphs
        budget = max(per_page, int((free - reserve) * opts.memory_fraction))
        return max(16, min(want * 2, budget // per_page))

    # ------------------------------------------------------------------ requests
    def add_request(self, prompt: Sequence[int], max_new_tokens: int, sampling: SamplingParameters = None,
                    stop_ids: Iterable[int] = (), rid: Optional[int] = None, deadline_s: Optional[float] = None,
                    cache_scope: bytes = b"", use_prefix_cache: bool = True, arrival: Optional[float] = None,
                    context_ceiling: Optional[int] = None) -> int:
        if rid is None:
            rid = self._next_rid
            self._next_rid += 1
        sampling = sampling or SamplingParameters()
        now = self.clock()
        # plain ints in a tuple: a tuple of ints is not tracked by the cyclic
        # garbage collector, so a long queue of prompts adds nothing to a pass
        toks = tuple(prompt.tolist() if hasattr(prompt, "tolist") else [int(t) for t in prompt])
        check_token_ids(toks, self.spec.vocab)
        req = Request(rid=rid, prompt=toks, max_new=max_new_tokens, sampling=sampling,
                      stop_ids=frozenset(int(t) for t in stop_ids),
                      deadline=None if deadline_s is None else now + deadline_s, cache_scope=cache_scope,
                      cache_enabled=use_prefix_cache, arrival=arrival if arrival is not None else now,
                      **({} if context_ceiling is None else {"context_ceiling": context_ceiling}))
        self.scheduler.add_request(req)
        self.live[rid] = req
        self.metrics.requests.inc()
        return rid

    def submit(self, g: GenerateRequest) -> int:
        if g.input_tokens is None:
            raise ValueError("text requests must be tokenized by the service layer first")
        return self.add_request(g.input_tokens, g.max_new_tokens, g.sampling, g.stop.token_ids, rid=g.request_id,
                                deadline_s=None if g.deadline_millis is None else g.deadline_millis / 1000.0,
                                cache_scope=g.cache.scope, use_prefix_cache=g.cache.permission.value != 0,
                                context_ceiling=g.context_ceiling)

    def cancel(self, rid: int) -> bool:
        ok = self.scheduler.cancel(rid)
        self._drain_terminals()
        return ok

    def has_work(self) -> bool:
        return self.scheduler.has_work()

    # ------------------------------------------------------------------ loop
    def step(self) -> List[TokenOutput]:
        """One engine step.  Synchronous by default: plan, run, commit.  With
        ``overlap_steps`` the next plan is built and launched while the
        previous step still runs (its decode rows take the pending tokens on
        the device), and then the previous step is committed, so host work
        of step n+1 hides behind the device time of step n."""
        if self.opts.overlap_steps:
            return self._step_overlap()
        t0 = self.clock()
        plan = self.scheduler.schedule()
        if plan is None:
            self._drain_terminals()
            return []
        self._observe_queue(plan, t0)
        try:
            sampled = self.runner.execute(plan, self.scheduler.tables.matrix)
        except Exception:
            # a device error word, or a launch that raised: the step's work is
            # void; active requests fail (retryably), waiting ones stay queued
            self._fail(plan)
            raise
        return self._commit(plan, sampled, t0)

    def _step_overlap(self) -> List[TokenOutput]:
        t0 = self.clock()
        plan = self.scheduler.schedule()
        if plan is not None:
            self._observe_queue(plan, t0)
            try:
                handle = self.runner.launch(plan, self.scheduler.tables.matrix)
            except Exception:
                self._fail(self._launched[0][0] if self._launched else plan)
                raise
            self._launched.append((plan, handle, t0))
        if not self._launched:
            self._drain_terminals()
            return []
        if plan is not None and len(self._launched) < 2:
            return []          # the first step of a burst: nothing to commit yet
        old, handle, ts = self._launched.pop(0)
        try:
            sampled = self.runner.wait(handle)
        except Exception:
            self._fail(old)
            raise
        return self._commit(old, sampled, ts)

    def _fail(self, plan):
        self._launched = []
        self.scheduler.abort_plan(plan)
        # the worker's step failed, not the request: retryable, as a lost rank is
        self.scheduler.fail_active(PublicErrorCode.WORKER_UNAVAILABLE)
        self._drain_terminals()

    def _observe_queue(self, plan, t0):
        for r in plan.rows:
            if not r.decode and r.start == r.req.cached_tokens:
                self.metrics.queue.observe(t0 - r.req.arrival)        # first step of this request

    def _commit(self, plan, sampled, t0) -> List[TokenOutput]:
        m = self.metrics
        outs = self.scheduler.complete(plan, sampled)
        for cb in self.listeners:
            cb(outs)
        self._drain_terminals()
        t1 = self.clock()
        kind = "prefill" if plan.prefill_rows else "decode"
        m.step_time.observe(t1 - t0, kind=kind)
        m.step_tokens.observe(plan.num_tokens)
        m.step_rows.observe(len(plan.rows))
        m.graph.inc(mode="captured" if self.runner.last_bucket is not None else "eager")
        for seconds in self.runner.take_capture_times():      # in steps or ahead of them
            m.graph_capture.observe(seconds)
        if outs:
            m.output_tokens.inc(len(outs))
            if m._last_emit is not None:
                m.itl.observe(t1 - m._last_emit)
            m._last_emit = t1
        a = self.scheduler.allocator
        m.kv_pages.set(a.free_page_count(), state="free")
        m.kv_pages.set(a.allocated_page_count(), state="allocated")
        return outs

    def _drain_terminals(self):
        for t in self.scheduler.take_terminals():
            req = self.live.pop(t.rid, None)
            if req is None:
                continue
            res = self.results[t.rid] = RequestResult(req.rid, len(req.prompt), list(req.output), t.reason, t.error,
                                                      req.arrival, req.first_token_time, req.finish_time,
                                                      req.cached_tokens)
            m = self.metrics
            if t.error is not None:
                m.failed.inc(code=t.error.name.lower())
            else:
                m.finished.inc(reason=t.reason.name.lower() if t.reason is not None else "none")
            m.prompt_tokens.inc(res.prompt_len)
            m.cached_tokens.inc(res.cached_tokens)
            if res.ttft is not None:
                m.ttft.observe(res.ttft)
            if res.tpot is not None:
                m.tpot.observe(res.tpot)

    def run_until_done(self, max_steps: int = 1 << 30):
        n = 0
        while self.has_work() and n < max_steps:
            self.step()
            n += 1
        return n

    # ------------------------------------------------------------------ public API
    def generate(self, prompts: Union[Sequence[Sequence[int]], torch.Tensor], max_new_tokens: int,
                 sampling: Optional[SamplingParameters] = None, seeds: Optional[Sequence[int]] = None
                 ) -> List[List[int]]:
        """Generates for a batch of token-id prompts (list of lists or a host
        int tensor [B, S], pinned for the fastest upload) and returns the
        generated ids per prompt."""
        if isinstance(prompts, torch.Tensor):
            arr = prompts.numpy()
            prompts = [arr[i] for i in range(arr.shape[0])]
        rids = []
        for i, p in enumerate(prompts):
            sp = sampling or SamplingParameters()
            if seeds is not None:
                sp = dataclasses.replace(sp, seed=int(seeds[i]))
            rids.append(self.add_request(p, max_new_tokens, sp))
        self.run_until_done()
        return [self.results.pop(r).tokens for r in rids]
