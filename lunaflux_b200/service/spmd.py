"""Tensor-parallel serving: one process per GPU, rank 0 at the front.

Rank 0 runs the service (TCP / HTTP endpoints, tokenizer, detokenisation)
on an engine wrapped by ``SpmdLeader``; every other rank runs
``follower_loop`` on its own engine shard.  All ranks run the same
deterministic scheduler, so the only thing that crosses is what changes it:
before each engine iteration the leader broadcasts the engine calls it made
since the previous one (requests added, requests cancelled), the clock value
the schedulers must see, and whether to step.  The followers replay the calls
and step in lock step; the kernels of a step then meet in their own
collectives.  No step plan is shipped.  The reference plans a worker that
receives step plans from the front (engine/device_worker); here the plan is
recomputed on every rank.

The broadcast uses the gloo control group (``torch.distributed``), so it
never touches the GPU stream.  While idle the leader broadcasts an empty
message on every wake-up of the service loop, which keeps the followers'
waits short of the group's timeout.
"""
from __future__ import annotations

import time
from typing import Callable, List, Optional

import torch.distributed as dist


class SharedClock:
    """The engines' clock on every rank: the leader's monotonic time, as
    broadcast with each iteration."""

    def __init__(self):
        self.now = time.monotonic()

    def __call__(self) -> float:
        return self.now


def _broadcast(msg, group):
    box = [msg]
    dist.broadcast_object_list(box, src=0, group=group)
    return box[0]


class SpmdLeader:
    """Rank 0's engine: forwards every call to the local engine and logs the
    ones that change the schedulers, for the next broadcast."""

    def __init__(self, engine, clock: SharedClock, group=None):
        self._engine = engine
        self._clock = clock
        self._group = group
        self._log: List[tuple] = []

    def __getattr__(self, name):
        return getattr(self._engine, name)

    def add_request(self, prompt, max_new_tokens, sampling=None, stop_ids=(), rid=None, deadline_s=None,
                    cache_scope=b"", use_prefix_cache=True, arrival=None, context_ceiling=None):
        self._clock.now = time.monotonic()
        rid = self._engine.add_request(prompt, max_new_tokens, sampling, stop_ids, rid, deadline_s, cache_scope,
                                       use_prefix_cache, arrival, context_ceiling)
        self._log.append(("add", (list(prompt), max_new_tokens, sampling, tuple(stop_ids), rid, deadline_s,
                                  cache_scope, use_prefix_cache, self._clock.now, context_ceiling)))
        return rid

    def submit(self, g):
        # the engine's own submit funnels into add_request
        return type(self._engine).submit(self, g)

    def cancel(self, rid: int) -> bool:
        self._log.append(("cancel", rid))
        return self._engine.cancel(rid)

    def _publish(self, step: bool):
        self._clock.now = time.monotonic()
        log, self._log = self._log, []
        _broadcast((self._clock.now, log, step), self._group)

    def step(self):
        self._publish(True)
        return self._engine.step()

    def idle(self):
        """Called by the service loop when it does not step."""
        self._publish(False)

    def shutdown(self):
        _broadcast(None, self._group)


def follower_loop(engine, clock: SharedClock, group=None, on_step: Optional[Callable] = None):
    """Replays the leader's calls and steps in lock step until it shuts down."""
    while True:
        msg = _broadcast(None, group)
        if msg is None:
            return
        now, log, step = msg
        for kind, payload in log:
            if kind == "add":
                prompt, max_new, sampling, stop_ids, rid, deadline_s, scope, use_prefix, t_add, ceiling = payload
                clock.now = t_add
                engine.add_request(prompt, max_new, sampling, stop_ids, rid, deadline_s, scope, use_prefix,
                                   context_ceiling=ceiling)
            else:
                engine.cancel(payload)
        clock.now = now
        if step:
            engine.step()
            if on_step is not None:
                on_step()
