"""Deterministic continuous-batching scheduler.

Reference: scheduler/core (planning.mbt:35-195 select_rows, :403-499
build_next; completion_commit.mbt:32-178; lifecycle.mbt:5-416;
admission.mbt:2-278).  Policy kept from the reference:

* decode-first: every running decode request gets its row before any prefill;
* chunked prefill inside ``step_token_budget`` (``prefill_chunk_tokens`` per
  row), prefill rows serialised before decode rows in the plan;
* an emergency page reserve that new admissions may not consume, so running
  decodes keep growing;
* FIFO admission with bounded aging (a request that waited more than
  ``waiting_age_threshold_steps`` steps is admitted before partial prefills);
* transactional planning: allocator / block-table checkpoints are rolled
  back if building a plan fails;
* intermediate prefill never samples; the final prefill chunk returns the
  first token; decode returns the next;
* stop token / max-output / context-ceiling terminals, cancellation and
  deadlines with a global request generation so stale completions are
  ignored; worker-failure drain fails active requests and keeps waiting ones.

Changed for B200 serving: up to ``max_active_requests`` rows per step (the
reference's production plan admits one), recompute-preemption when pages run
out, and radix prefix reuse at admission (full pages only; pages of finished
requests are published into the cache).
"""
from __future__ import annotations

import collections
import dataclasses
import time
from typing import Callable, Deque, Dict, List, Optional, Sequence, Tuple

import numpy as np

from ..contracts import (FinishReason, PublicErrorCode, RequestState, SamplingMode, SamplingParameters,
                         can_transition)
from ..config import CacheConfig, SchedulerConfig
from ..kv.block_table import BlockTableArena, TableId
from ..kv.page_allocator import OutOfPages, PageAllocator, PageId
from ..prefix.radix import PrefixIdentity, PrefixIndex


_TERMINAL_STATES = frozenset(st for st in RequestState if st.terminal)


class SchedulerError(RuntimeError):
    pass


class AdmissionRejected(SchedulerError):
    def __init__(self, code: PublicErrorCode, why: str):
        super().__init__(why)
        self.code = code


@dataclasses.dataclass(eq=False)
class Request:
    rid: int
    prompt: List[int]
    max_new: int
    sampling: SamplingParameters
    stop_ids: frozenset = frozenset()
    context_ceiling: int = 1 << 30
    deadline: Optional[float] = None
    cache_scope: bytes = b""
    cache_enabled: bool = True
    arrival: float = 0.0
    # mutable scheduler state
    state: RequestState = RequestState.WAITING
    generation: int = 0
    table: Optional[TableId] = None
    pages: List[PageId] = dataclasses.field(default_factory=list)
    num_computed: int = 0
    # Planning state, ahead of num_computed / output while steps are in
    # flight: the KV length once every scheduled row has run, the sampled
    # tokens not yet returned, and where the newest of them sits in its
    # step's sampling order (its next decode row reads it on the device).
    sched_len: int = 0
    pending: int = 0
    pending_slot: int = -1
    cached_tokens: int = 0
    output: List[int] = dataclasses.field(default_factory=list)
    prefix_nodes: list = dataclasses.field(default_factory=list)
    enqueued_step: int = 0
    first_token_time: Optional[float] = None
    last_token_time: Optional[float] = None
    finish_time: Optional[float] = None
    finish_reason: Optional[FinishReason] = None
    error: Optional[PublicErrorCode] = None
    preemptions: int = 0

    @property
    def total_len(self) -> int:
        return len(self.prompt) + len(self.output)

    def token_at(self, i: int) -> int:
        n = len(self.prompt)
        return self.prompt[i] if i < n else self.output[i - n]

    def tokens_upto(self, n: int) -> List[int]:
        """The first n tokens of prompt + output, as one list (slices, no per-token calls)."""
        p = self.prompt
        if n <= len(p):
            return list(p[:n])
        return list(p) + list(self.output[: n - len(p)])

    @property
    def prefill_target(self) -> int:
        """KV length at which prefill ends (the whole prompt, or after a
        preemption everything except the last sampled token)."""
        return self.total_len - 1 if self.output else len(self.prompt)


@dataclasses.dataclass
class Row:
    req: Request
    start: int            # first position (== KV length before the step)
    n: int                # tokens in the row
    sample: bool          # whether the row produces a token
    decode: bool
    generation: int
    sample_index: int = 0     # index of the sampled token in the request's output
    fwd: int = -1             # decode input taken on the device from the previous step's sample slot


@dataclasses.dataclass
class StepPlan:
    seq: int
    rows: List[Row]       # prefill rows first, then decode rows

    @property
    def num_tokens(self) -> int:
        return sum(r.n for r in self.rows)

    @property
    def prefill_rows(self) -> List[Row]:
        return [r for r in self.rows if not r.decode]

    @property
    def decode_rows(self) -> List[Row]:
        return [r for r in self.rows if r.decode]

    @property
    def sample_rows(self) -> List[Row]:
        return [r for r in self.rows if r.sample]


@dataclasses.dataclass
class TokenOutput:
    rid: int
    token: int
    position: int
    finished: bool
    reason: Optional[FinishReason]


@dataclasses.dataclass
class Terminal:
    rid: int
    reason: Optional[FinishReason]
    error: Optional[PublicErrorCode]


class Scheduler:
    def __init__(self, cfg: SchedulerConfig, cache: CacheConfig, num_pages: int, identity: Optional[PrefixIdentity] = None,
                 clock: Callable[[], float] = time.monotonic, max_context: int = 8192, first_page: int = 1):
        self.cfg = cfg
        self.cache_cfg = cache
        self.P = cache.tokens_per_page
        self.clock = clock
        self.max_context = max_context
        self.pages_per_request = min(cache.block_table_pages_per_request, -(-max_context // self.P))
        self.allocator = PageAllocator(num_pages, first_index=first_page)
        self.tables = BlockTableArena(cfg.max_active_requests, self.pages_per_request, self.P)
        self.identity = identity
        self.prefix = PrefixIndex(self.allocator, self.P, cache.prefix_max_pages) if (
            cache.prefix_enabled and identity is not None) else None
        self.requests: Dict[int, Request] = {}
        self.waiting: Deque[Request] = collections.deque()
        self.running: List[Request] = []
        self.step_seq = 0
        self.generation = 0
        self.terminals: List[Terminal] = []
        # Plans handed to the device and not yet completed, oldest first.  With
        # max_inflight = 2 the next step is planned while the current one runs:
        # its decode rows read the pending tokens on the device.
        self.inflight: List[StepPlan] = []
        self.max_inflight = 1
        # metrics
        self.preemptions = 0
        self.prompt_tokens_computed = 0
        self.prefix_hit_tokens = 0

    # ------------------------------------------------------------------ admission
    def add_request(self, req: Request):
        if req.rid in self.requests:
            raise AdmissionRejected(PublicErrorCode.INVALID_REQUEST, "duplicate live request id")
        if len(self.waiting) >= self.cfg.max_waiting_requests:
            raise AdmissionRejected(PublicErrorCode.OVERLOADED, "waiting queue full")
        ceiling = min(req.context_ceiling, self.max_context, self.pages_per_request * self.P)
        if len(req.prompt) == 0 or len(req.prompt) >= ceiling:
            raise AdmissionRejected(PublicErrorCode.CONTEXT_OVERFLOW, "prompt does not fit the context")
        if -(-len(req.prompt) // self.P) + 1 > self.allocator.capacity:
            raise AdmissionRejected(PublicErrorCode.CONTEXT_OVERFLOW, "prompt exceeds the KV arena")
        req.context_ceiling = ceiling
        self.generation += 1
        req.generation = self.generation
        req.state = RequestState.WAITING
        req.enqueued_step = self.step_seq
        if not req.arrival:
            req.arrival = self.clock()
        self.requests[req.rid] = req
        self.waiting.append(req)

    def has_work(self) -> bool:
        return bool(self.waiting or self.running or self.inflight)

    # ------------------------------------------------------------------ lifecycle
    def cancel(self, rid: int) -> bool:
        req = self.requests.get(rid)
        if req is None or req.state.terminal:
            return False
        self.generation += 1
        req.generation = self.generation
        self._finish(req, RequestState.CANCELLED, FinishReason.CANCELLED, None)
        return True

    def expire_deadlines(self):
        now = self.clock()
        for req in list(self.waiting) + list(self.running):
            if req.deadline is not None and now >= req.deadline and not req.state.terminal:
                self.generation += 1
                req.generation = self.generation
                self._finish(req, RequestState.FAILED, None, PublicErrorCode.DEADLINE_EXCEEDED)

    def fail_active(self, code: PublicErrorCode = PublicErrorCode.WORKER_UNAVAILABLE):
        """Worker loss: fail every request with device state; waiting ones survive."""
        for req in list(self.running):
            self.generation += 1
            req.generation = self.generation
            self._finish(req, RequestState.FAILED, None, code)
        self.inflight = []

    def take_terminals(self) -> List[Terminal]:
        t, self.terminals = self.terminals, []
        return t

    def _release_kv(self, req: Request, publish: bool):
        if req.table is None:
            return
        if publish and self.prefix is not None and req.cache_enabled:
            n_full = req.num_computed // self.P
            if n_full:
                toks = req.tokens_upto(n_full * self.P)
                self.prefix.insert(self._ident(req), toks, req.pages[:n_full])
        if req.prefix_nodes:
            self.prefix.release(req.prefix_nodes)
            req.prefix_nodes = []
        self.tables.reset_and_release(req.table, self.allocator)
        req.table = None
        req.pages = []

    def _ident(self, req: Request) -> PrefixIdentity:
        i = self.identity
        return PrefixIdentity(i.model_digest, i.tokenizer_digest, req.cache_scope, i.tokens_per_page,
                              i.layout_version)

    def _finish(self, req: Request, state: RequestState, reason, error):
        if req in self.running:
            self.running.remove(req)
        elif req in self.waiting:
            self.waiting.remove(req)
        self._release_kv(req, publish=(state is RequestState.FINISHED))
        req.state = state
        req.finish_reason = reason
        req.error = error
        req.finish_time = self.clock()
        self.terminals.append(Terminal(req.rid, reason, error))
        self.requests.pop(req.rid, None)

    # ------------------------------------------------------------------ planning
    def _pages_needed(self, req: Request, upto: int) -> int:
        return max(0, -(-upto // self.P) - len(req.pages))

    def _grow(self, req: Request, upto: int):
        need = self._pages_needed(req, upto)
        if need:
            pids = self.allocator.allocate_run(need)
            self.tables.note(req.table)
            self.tables.append_pages(req.table, pids)
            req.pages.extend(pids)

    def _make_room(self, need: int, protect: Request) -> bool:
        """Frees pages by prefix eviction, then recompute-preemption of the
        newest running request.  Returns False if nothing more can be freed."""
        while self.allocator.free_page_count() < need:
            if self.prefix is not None and self.prefix.evict(need - self.allocator.free_page_count()) > 0:
                continue
            victim = next((r for r in reversed(self.running) if r is not protect), None)
            if victim is None:
                return False
            self._preempt(victim)
        return True

    def _preempt(self, req: Request):
        self.running.remove(req)
        self._release_kv(req, publish=False)
        # Rows of this request still in flight become stale and their tokens
        # are recomputed after re-admission.  Its pages may go to a request of
        # a later plan: that plan runs after the in-flight one on the same
        # stream, so the stale writes land first and are overwritten.
        self.generation += 1
        req.generation = self.generation
        req.pending = 0
        req.pending_slot = -1
        req.sched_len = 0
        req.num_computed = 0
        req.cached_tokens = 0
        req.state = RequestState.WAITING
        req.preemptions += 1
        self.preemptions += 1
        self.waiting.appendleft(req)

    def _admit(self, req: Request) -> bool:
        """Moves a waiting request to running with a block table and any
        prefix-cache pages.  Returns False if no table is free."""
        if self.tables.free_table_count() == 0:
            return False
        req.table = self.tables.allocate()
        req.pages = []
        req.num_computed = 0
        req.sched_len = 0
        if self.prefix is not None and req.cache_enabled:
            seq_len = req.prefill_target
            toks = req.tokens_upto(seq_len)
            # keep at least one token to compute so the row produces logits
            nodes = self.prefix.lookup(self._ident(req), toks, max_pages=(seq_len - 1) // self.P)
            if nodes:
                self.prefix.retain(nodes)
                req.prefix_nodes = nodes
                pids = self.prefix.pages_of(nodes)
                for p in pids:
                    self.allocator.retain_active(p)
                self.tables.append_pages(req.table, pids)
                req.pages = pids
                req.num_computed = len(pids) * self.P
                req.sched_len = req.num_computed
                req.cached_tokens = req.num_computed
                self.prefix_hit_tokens += req.num_computed
        self.waiting.remove(req)
        self.running.append(req)
        req.state = RequestState.PREFILL
        return True

    def schedule(self) -> Optional[StepPlan]:
        """Builds the next step plan (None when idle)."""
        if len(self.inflight) >= self.max_inflight:
            raise SchedulerError("previous plan not completed")
        self.expire_deadlines()
        if not self.running and not self.waiting:
            return None
        rows = self._plan_rows(admit=True)
        while not rows and self.running and not self.inflight:
            # Every running request is blocked on KV pages (none can take a
            # row) and nothing in flight will free any: recompute the youngest
            # (its pages go to the older ones), or fail a request that cannot
            # fit the cache on its own.  No admission during the retry, so the
            # freed pages reach the requests already running.
            if len(self.running) > 1:
                self._preempt(self.running[-1])
            else:
                req = self.running[0]
                self.generation += 1
                req.generation = self.generation
                self._finish(req, RequestState.FAILED, None, PublicErrorCode.CONTEXT_OVERFLOW)
            rows = self._plan_rows(admit=False)
        if not rows:
            return None
        # advance the planning state (the committed state moves on completion)
        slot = 0
        for r in rows:
            req = r.req
            req.sched_len = r.start + r.n
            if not r.decode and req.sched_len == req.prefill_target:
                req.state = RequestState.DECODE
            if r.sample:
                r.sample_index = len(req.output) + req.pending
                req.pending += 1
                req.pending_slot = slot
                slot += 1
        self.step_seq += 1
        plan = StepPlan(self.step_seq, rows)
        self.inflight.append(plan)
        return plan

    def _plan_rows(self, admit: bool) -> List[Row]:
        """Decode rows, then prefill chunks, within the step budget (KV pages
        allocated as rows are chosen); waiting requests are admitted only when
        ``admit``."""
        cfg = self.cfg
        budget = cfg.step_token_budget
        max_rows = cfg.max_rows_per_step
        decode_rows: List[Row] = []
        prefill_rows: List[Row] = []

        # 1. decode-first
        # (a request preempted below to make room leaves DECODE for WAITING)
        decoding = RequestState.DECODE
        for req in list(self.running):
            if req.state is not decoding:
                continue
            if len(decode_rows) >= max_rows or budget <= 0:
                break
            produced = len(req.output) + req.pending
            if produced >= req.max_new or len(req.prompt) + produced >= req.context_ceiling:
                continue        # its last token is still in flight; it finishes on completion
            need = self._pages_needed(req, req.sched_len + 1)
            if need and not self._make_room(need, req):
                continue
            self._grow(req, req.sched_len + 1)
            decode_rows.append(Row(req, req.sched_len, 1, True, True, req.generation,
                                   fwd=req.pending_slot if req.pending else -1))
            budget -= 1
        # drop rows whose request was preempted while making room for a later one
        decode_rows = [r for r in decode_rows if r.req.state is decoding]

        # 2. prefill: aged waiting requests, then partial prefills, then FIFO waiting
        rows_used = len(decode_rows)
        reserve = cfg.emergency_decode_page_reserve
        aged: List[Request] = []
        fresh: List[Request] = []
        if admit:     # one pass over the queue (it can hold thousands of requests)
            cut = self.step_seq - cfg.waiting_age_threshold_steps
            for r in self.waiting:
                (aged if r.enqueued_step <= cut else fresh).append(r)
        partial = [r for r in self.running if r.state is RequestState.PREFILL]
        for req in aged + partial + fresh:
            if budget <= 0 or rows_used >= max_rows:
                break
            is_new = req.state is RequestState.WAITING
            if is_new:
                # admission must leave the emergency reserve untouched
                first_chunk = min(req.prefill_target, cfg.prefill_chunk_tokens, budget)
                if self.allocator.free_page_count() - (-(-first_chunk // self.P)) < reserve and self.running:
                    if self.prefix is None or self.prefix.evict(reserve) == 0:
                        break
                if not self._admit(req):
                    break
            chunk = min(req.prefill_target - req.sched_len, cfg.prefill_chunk_tokens, budget)
            if chunk <= 0:
                continue
            need = self._pages_needed(req, req.sched_len + chunk)
            if need > self.allocator.free_page_count():
                if self.prefix is not None:
                    self.prefix.evict(need - self.allocator.free_page_count())
                if need > self.allocator.free_page_count():
                    chunk = (len(req.pages) + self.allocator.free_page_count()) * self.P - req.sched_len
                    if chunk <= 0:
                        if is_new:
                            self._preempt_new(req)
                        break
            self._grow(req, req.sched_len + chunk)
            final = req.sched_len + chunk == req.prefill_target
            prefill_rows.append(Row(req, req.sched_len, chunk, final and not req.output, False, req.generation))
            budget -= chunk
            rows_used += 1

        return prefill_rows + decode_rows

    def _preempt_new(self, req: Request):
        self.running.remove(req)
        self._release_kv(req, publish=False)
        req.sched_len = 0
        req.state = RequestState.WAITING
        self.waiting.appendleft(req)

    # ------------------------------------------------------------------ completion
    def complete(self, plan: StepPlan, sampled: Sequence[int]) -> List[TokenOutput]:
        """Commits a finished step: ``sampled[i]`` is the token of the i-th
        sampling row, in plan order."""
        if not self.inflight or self.inflight[0] is not plan:
            raise SchedulerError("completion for a plan that is not the oldest in flight")
        n_sample = sum(1 for r in plan.rows if r.sample)
        if len(sampled) != n_sample:
            # checked before anything moves: the plan stays in flight for a correct retry
            raise SchedulerError(f"completion carries {len(sampled)} tokens for {n_sample} sampling rows")
        self.inflight.pop(0)
        now = self.clock()
        outs: List[TokenOutput] = []
        append = outs.append
        toks = [int(t) for t in sampled]
        terminal = _TERMINAL_STATES
        si = 0
        for row in plan.rows:
            tok = None
            if row.sample:
                tok = toks[si]
                si += 1
            req = row.req
            if req.generation != row.generation or req.state in terminal:
                continue  # stale: cancelled / expired while in flight
            req.num_computed = row.start + row.n
            if not row.decode:
                self.prompt_tokens_computed += row.n
            if tok is None:
                continue
            req.pending -= 1
            out = req.output
            out.append(tok)
            if req.first_token_time is None:
                req.first_token_time = now
            req.last_token_time = now
            total = len(req.prompt) + len(out)
            reason = None
            if tok in req.stop_ids:
                reason = FinishReason.STOP_SEQUENCE
            elif len(out) >= req.max_new or total >= req.context_ceiling:
                reason = FinishReason.TOKEN_LIMIT
            append(TokenOutput(req.rid, tok, total - 1, reason is not None, reason))
            if reason is not None:
                self._finish(req, RequestState.FINISHED, reason, None)
        return outs

    def abort_plan(self, plan: StepPlan):
        """The step failed on the device: the plan (and any planned after it)
        is dropped; the caller fails the active requests."""
        if plan in self.inflight:
            self.inflight = self.inflight[:self.inflight.index(plan)]

    # ------------------------------------------------------------------ diagnostics
    def debug_check_invariants(self):
        self.allocator.debug_check_invariants()
        for req in self.running:
            assert req.table is not None
            assert len(req.pages) == self.tables.page_count(req.table)
            assert len(req.pages) * self.P >= req.num_computed
            for p in req.pages:
                assert self.allocator.validate_active(p)
        for req in self.waiting:
            assert req.table is None and not req.pages
        if self.prefix is not None:
            self.prefix.debug_check_invariants()
