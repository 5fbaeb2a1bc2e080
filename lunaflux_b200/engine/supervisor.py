"""Rank supervisor: one worker process per GPU, heartbeats, ordered recovery.

Reference: engine/worker_process (supervisor.mbt:129-257, root_bound.mbt:167-480:
Configure -> Ready handshake, one outstanding plan, ordered recovery: close /
reap the child, retire what completed, fail what was submitted, start a
replacement with a new generation) and engine/worker_service/README.mbt.md:93-114
(worker failure fails device-backed requests, waiting requests survive).

Here the workers are the ranks of one tensor-parallel group.  Every rank runs
the same deterministic engine; the supervisor sends every rank the same
command stream (admissions, cancellations, "step"), so the ranks stay in lock
step without broadcasting plans.  Each rank reports its outputs (rank 0's are
authoritative) and sends a heartbeat every ``heartbeat_s``.  A rank that
exits, closes its channel, raises, or misses heartbeats for ``dead_after_s``
fails the generation: every rank is terminated and reaped, requests that had
produced tokens fail with ``worker_unavailable`` (retryable), requests that had
not are re-submitted to the next generation, which is started fresh.

The control channel is a socketpair carrying framed, checksummed messages
(``engine/channel.py``: the C++ channel core with exact I/O and deadlines);
the GPU data path never crosses it.
"""
from __future__ import annotations

import dataclasses
import multiprocessing as mp
import os
import select
import socket
import threading
import time
import traceback
from typing import Callable, Dict, List, Optional, Tuple

from ..contracts import PublicErrorCode
from .channel import MessageChannel


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank_main(rank: int, world: int, port: int, factory: Callable, sock, heartbeat_s: float, generation: int):
    """Worker process body: build the engine, then serve the command stream."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), LUNAFLUX_GENERATION=str(generation))
    conn = MessageChannel(sock)
    conn.generation = generation
    stop = threading.Event()

    def send(msg):
        conn.send(msg)  # the channel serialises concurrent senders

    def beat():
        while not stop.is_set():
            try:
                send(("hb", rank, time.monotonic()))
            except (OSError, BrokenPipeError, EOFError):
                return
            stop.wait(heartbeat_s)

    threading.Thread(target=beat, daemon=True).start()
    try:
        engine = factory(rank, world)
        send(("ready", rank))
        while True:
            msg = conn.recv(1.0)
            if msg is None:
                continue
            kind = msg[0]
            if kind == "add":
                _, rid, prompt, max_new, sampling, stop_ids = msg
                engine.add_request(prompt, max_new, sampling, stop_ids, rid=rid)
            elif kind == "cancel":
                engine.cancel(msg[1])
            elif kind == "step":
                shared = getattr(engine, "shared_clock", None)
                if shared is not None:
                    shared.now = msg[1]    # every rank's scheduler sees the supervisor's clock
                outs = engine.step()
                done = [(rid, r.reason.name if r.reason else None, r.error.name if r.error else None)
                        for rid, r in list(engine.results.items())]
                engine.results.clear()
                send(("outs", rank, [(o.rid, o.token, o.finished) for o in outs], done, engine.has_work()))
            elif kind == "close":
                break
    except (EOFError, OSError):
        pass
    except Exception:
        try:
            send(("error", rank, traceback.format_exc(limit=5)))
        except Exception:
            pass
    finally:
        stop.set()


@dataclasses.dataclass
class _Req:
    rid: int
    prompt: List[int]
    max_new: int
    sampling: object
    stop_ids: Tuple[int, ...]
    tokens: List[int] = dataclasses.field(default_factory=list)
    done: bool = False
    reason: Optional[str] = None
    error: Optional[PublicErrorCode] = None


class WorkerLost(RuntimeError):
    pass


class Supervisor:
    def __init__(self, world: int, factory: Callable, heartbeat_s: float = 0.2, dead_after_s: float = 5.0,
                 step_timeout_s: float = 60.0, start_method: str = "spawn"):
        self.world = world
        self.factory = factory
        self.heartbeat_s = heartbeat_s
        self.dead_after_s = dead_after_s
        self.step_timeout_s = step_timeout_s
        self.ctx = mp.get_context(start_method)
        self.generation = 0
        self.procs: List = []
        self.conns: List = []
        self.last_beat: Dict[int, float] = {}
        self.reqs: Dict[int, _Req] = {}
        self.failures = 0
        self.ready = set()
        self.last_outs: List = []      # rank 0's (rid, token, finished) of the last step
        self.last_done: List = []      # rank 0's (rid, reason, error) terminals of the last step
        self.last_failed: List[int] = []   # requests failed by the last recovery

    # ------------------------------------------------------------------ lifecycle
    def start(self):
        self.generation += 1
        port = _free_port()
        self.procs, self.conns = [], []
        for r in range(self.world):
            parent, child = socket.socketpair()
            p = self.ctx.Process(target=_rank_main, args=(r, self.world, port, self.factory, child, self.heartbeat_s,
                                                          self.generation), daemon=True)
            p.start()
            child.close()
            self.procs.append(p)
            conn = MessageChannel(parent)
            conn.generation = self.generation    # frames of another generation are rejected
            self.conns.append(conn)
        now = time.monotonic()
        self.last_beat = {r: now for r in range(self.world)}
        self.ready = set()  # heartbeats are checked once a rank has finished starting
        deadline = now + self.step_timeout_s
        try:
            while len(self.ready) < self.world:
                for r, msg in self._poll(deadline):
                    if msg[0] == "ready":
                        self.ready.add(r)
                        self.last_beat[r] = time.monotonic()
        except WorkerLost:
            # a rank that cannot start fails the whole start: no rank of this
            # generation is left running
            self._reap()
            raise
        # re-submit requests that were waiting when the previous generation died
        for q in self.reqs.values():
            if not q.done:
                self._send_all(("add", q.rid, q.prompt, q.max_new, q.sampling, q.stop_ids))

    def close(self):
        for c in self.conns:
            try:
                c.send(("close",))
            except Exception:
                pass
        self._reap(graceful=True)

    def _reap(self, graceful: bool = False):
        for p in self.procs:
            p.join(timeout=5 if graceful else 0.5)
            if p.is_alive():
                p.terminate()
                p.join(timeout=5)
            if p.is_alive():
                p.kill()
                p.join(timeout=5)
        for c in self.conns:
            try:
                c.close()
            except Exception:
                pass
        self.procs, self.conns = [], []

    # ------------------------------------------------------------------ channel
    def _send_all(self, msg):
        for r, c in enumerate(self.conns):
            try:
                c.send(msg)
            except (OSError, BrokenPipeError):
                raise WorkerLost(f"rank {r} channel closed")

    def _poll(self, deadline: float):
        """Yields (rank, message) until the deadline; raises WorkerLost on a dead rank."""
        got = []
        while not got:
            now = time.monotonic()
            for r, p in enumerate(self.procs):
                if not p.is_alive():
                    raise WorkerLost(f"rank {r} exited ({p.exitcode})")
                if r in self.ready and now - self.last_beat.get(r, now) > self.dead_after_s:
                    raise WorkerLost(f"rank {r} missed heartbeats")
            if now > deadline:
                raise WorkerLost("step timed out")
            ready = select.select(self.conns, [], [], min(0.05, self.heartbeat_s))[0]
            for c in ready:
                r = self.conns.index(c)
                try:
                    msg = c.recv(0.0)
                except (EOFError, OSError):
                    raise WorkerLost(f"rank {r} channel closed")
                if msg is None:
                    continue
                if msg[0] == "hb":
                    self.last_beat[r] = time.monotonic()
                elif msg[0] == "error":
                    raise WorkerLost(f"rank {r} raised: {msg[2].splitlines()[-1]}")
                else:
                    got.append((r, msg))
        return got

    # ------------------------------------------------------------------ API
    def submit(self, rid: int, prompt, max_new: int, sampling=None, stop_ids=()):
        from ..contracts import SamplingParameters
        q = _Req(rid, list(prompt), max_new, sampling or SamplingParameters(), tuple(stop_ids))
        self.reqs[rid] = q
        try:
            self._send_all(("add", rid, q.prompt, max_new, q.sampling, q.stop_ids))
        except WorkerLost:
            pass    # the next step finds the lost rank; recovery re-submits this request

    def cancel(self, rid: int):
        try:
            self._send_all(("cancel", rid))
        except WorkerLost:
            # the next step recovers; the request must not come back with it
            q = self.reqs.get(rid)
            if q is not None and not q.done:
                q.done, q.reason = True, "CANCELLED"

    def step(self) -> bool:
        """One engine iteration on every rank.  Returns whether work remains.
        A lost rank triggers recovery and returns True (the new generation
        continues with the surviving requests)."""
        try:
            self._send_all(("step", time.monotonic()))
            replies = {}
            deadline = time.monotonic() + self.step_timeout_s
            while len(replies) < self.world:
                for r, msg in self._poll(deadline):
                    if msg[0] == "outs":
                        replies[r] = msg
        except WorkerLost:
            self.last_outs, self.last_done = [], []
            self._recover()
            return True
        _, _, outs, done, more = replies[0]
        self.last_outs, self.last_done = outs, done
        for rid, tok, _fin in outs:
            if rid in self.reqs:
                self.reqs[rid].tokens.append(tok)
        for rid, reason, err in done:
            q = self.reqs.get(rid)
            if q is not None:
                q.done, q.reason = True, reason
                q.error = PublicErrorCode[err] if err else None
        return more

    def _recover(self):
        """Ordered recovery: reap every rank, fail requests that were producing
        tokens, keep the rest, start the next generation."""
        self.failures += 1
        self._reap()
        self.last_failed = []
        for q in self.reqs.values():
            if not q.done and q.tokens:
                q.done, q.error = True, PublicErrorCode.WORKER_UNAVAILABLE
                self.last_failed.append(q.rid)
        self.start()

    def run_until_done(self, max_steps: int = 100000):
        n = 0
        while any(not q.done for q in self.reqs.values()) and n < max_steps:
            self.step()
            n += 1
        return n
