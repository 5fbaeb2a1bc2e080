"""The serving loop and the framed TCP endpoint.

Reference: service/online_session (LunaOnlineInstance begin / progress /
take_event, admission.mbt:90, progression.mbt:225), service/online_tcp
(endpoint_prepare.mbt:53, endpoint_reactor.mbt:203), service/request_admission
(prepare_luna_request, admit.mbt:329).  Kept: the receipt time is the
monotonic time at which the request's first byte arrived (framed TCP) or the
connection was accepted (HTTP); the deadline is derived from it once, checked
before and after tokenization, and what is left of it goes to the scheduler;
the event order Accepted -> Token* -> Usage -> Completed | Failed; a worker
failure fails active requests with ``worker_unavailable`` (retryable);
draining rejects new admissions.  Changed: many concurrent connections and
requests (the reference serves one request on one connection), continuous
batching underneath, and client disconnect cancels the request.

Threads: the engine runs in one dedicated thread (it owns the GPU stream and
the scheduler); asyncio handles sockets; the two meet through a locked inbox
and ``call_soon_threadsafe``.
"""
from __future__ import annotations

import asyncio
import gc
import collections
import concurrent.futures
import threading
import time
from dataclasses import dataclass
from typing import Callable, Deque, Dict, Optional

from ..contracts.inference import (CompletedEvent, FailedEvent, FinishReason, GenerateRequest, InferenceLimits,
                                   PublicErrorCode, TokenEvent, Usage)
from ..engine.engine import LLMEngine
from ..scheduler.scheduler import AdmissionRejected
from ..tokenizer.bpe import Tokenizer
from .detokenize import IncrementalOutput
from .framed_wire import (REQUEST_MAGIC, AcceptedWire, FrameReader, FramedWireError, decode_request, encode_event)


@dataclass
class _Live:
    req: GenerateRequest
    sink: Callable[[object], None]
    out: IncrementalOutput
    prompt_len: int
    n_out: int = 0


def _guarded(sink: Callable[[object], None]) -> Callable[[object], None]:
    """A sink whose failure (a client's event loop already closed, a broken
    callback) drops that event instead of ending the engine thread."""
    def emit(ev):
        try:
            sink(ev)
        except Exception:
            pass
    return emit


class EngineService:
    """Owns the engine thread; thread-safe submit / cancel; events via sinks."""

    def __init__(self, engine: LLMEngine, tokenizer: Optional[Tokenizer], limits: InferenceLimits,
                 content_digest: str = "", plan_digest: str = "", tokenizer_threads: int = 2,
                 clock: Callable[[], float] = time.monotonic):
        self.engine = engine
        # receipt times and deadlines; the engine's scheduler gets the time left
        self.clock = clock
        self.tokenizer = tokenizer
        self.limits = limits
        self.content_digest = content_digest
        self.plan_digest = plan_digest or engine.spec.plan_digest()
        self._inbox: Deque = collections.deque()
        self._cv = threading.Condition()
        self._live: Dict[int, _Live] = {}
        self._stop = False
        self.draining = False
        self.failed = False
        self._thread = threading.Thread(target=self._run, name="lunaflux-engine", daemon=True)
        self._tok_pool = concurrent.futures.ThreadPoolExecutor(max_workers=tokenizer_threads,
                                                               thread_name_prefix="lunaflux-tokenizer")
        self.engine.listeners.append(self._on_outputs)

    def start(self):
        # Everything built so far (model, kernels, graphs, modules) lives as
        # long as the process: move it out of the collector's reach, so a full
        # collection during serving walks only the serving state (measured: a
        # full pass fell from ~94 ms to a few ms in a process with torch loaded).
        gc.collect()
        gc.freeze()
        self._thread.start()

    def alive(self) -> bool:
        """The engine loop runs and has not failed."""
        return self._thread.is_alive() and not self.failed and not self._stop

    def stop(self):
        with self._cv:
            self._stop = True
            self._cv.notify()
        self._thread.join(timeout=30)
        self._tok_pool.shutdown(wait=False, cancel_futures=True)

    # -------------------------------------------------------------- producer side
    def submit(self, req: GenerateRequest, sink: Callable[[object], None], receipt: Optional[float] = None):
        """Queues a request for the engine thread.  ``receipt`` is when the
        request arrived on this service's clock (now if not given); a
        request's ``deadline_millis`` counts from it.  Text prompts are
        tokenized first on the tokenizer pool, so a long prompt never stalls a
        step.  While draining, new requests are refused here (retryable
        ``overloaded``); those queued before the drain began are admitted."""
        if receipt is None:
            receipt = self.clock()
        sink = _guarded(sink)
        if self.draining:
            sink(FailedEvent(req.request_id, PublicErrorCode.OVERLOADED, True))
            return
        if self._expired(req, receipt, sink):
            return
        if req.input_text is not None and self.tokenizer is not None:
            self._tok_pool.submit(self._tokenize_then_queue, req, sink, receipt)
            return
        self._queue(req, sink, receipt)

    def _expired(self, req: GenerateRequest, receipt: float, sink) -> bool:
        if req.deadline_millis is not None and self.clock() >= receipt + req.deadline_millis / 1000.0:
            sink(FailedEvent(req.request_id, PublicErrorCode.DEADLINE_EXCEEDED, False))
            return True
        return False

    def _queue(self, req, sink, receipt):
        with self._cv:
            self._inbox.append(("add", (req, receipt), sink))
            self._cv.notify()

    def _tokenize_then_queue(self, req: GenerateRequest, sink, receipt: float):
        try:
            ids = tuple(self.tokenizer.encode_bytes(req.input_text, allow_special=False))
        except ValueError:
            sink(FailedEvent(req.request_id, PublicErrorCode.INVALID_REQUEST, False))
            return
        if not ids:
            sink(FailedEvent(req.request_id, PublicErrorCode.INVALID_REQUEST, False))
            return
        if self._expired(req, receipt, sink):
            return
        self._queue(GenerateRequest(**{**req.__dict__, "input_tokens": ids, "input_text": None}), sink, receipt)

    def cancel(self, rid: int):
        with self._cv:
            self._inbox.append(("cancel", rid, None))
            self._cv.notify()

    def drain(self, timeout_s: float, poll_s: float = 0.01) -> bool:
        """Graceful drain (the service configuration's graceful_drain_ms):
        new requests are refused from now on (retryable ``overloaded``), the
        live ones may finish for up to ``timeout_s``; whatever is still live
        then is cancelled in the engine and fails with the retryable
        ``worker_unavailable`` code.  Returns True when every live request
        finished in time.  Reference: config/service/service.mbt:39-107
        (graceful_drain_milliseconds) and the drain path of
        service/online_session."""
        self.draining = True
        deadline = time.monotonic() + max(0.0, timeout_s)
        while time.monotonic() < deadline:
            with self._cv:
                if not self._live and not self._inbox:
                    return True
            time.sleep(poll_s)
        with self._cv:
            if not self._live and not self._inbox:
                return True
            done = threading.Event()
            self._inbox.append(("drain_deadline", done, None))
            self._cv.notify()
        # the engine thread fails the remaining requests
        while not done.wait(poll_s) and self._thread.is_alive():
            pass
        return False

    # -------------------------------------------------------------- engine thread
    def _admit(self, req: GenerateRequest, receipt: float, sink):
        if self.failed:
            sink(FailedEvent(req.request_id, PublicErrorCode.WORKER_UNAVAILABLE, True))
            return
        if (req.model_content_digest and self.content_digest and req.model_content_digest != self.content_digest) or \
                (req.model_plan_digest and req.model_plan_digest != self.plan_digest):
            sink(FailedEvent(req.request_id, PublicErrorCode.INVALID_REQUEST, False))
            return
        if req.input_tokens is not None:
            prompt = list(req.input_tokens)
        else:
            if self.tokenizer is None:
                sink(FailedEvent(req.request_id, PublicErrorCode.INVALID_REQUEST, False))
                return
            try:
                prompt = self.tokenizer.encode_bytes(req.input_text, allow_special=False)
            except ValueError:
                sink(FailedEvent(req.request_id, PublicErrorCode.INVALID_REQUEST, False))
                return
        if not prompt or max(prompt) > self.limits.max_token_id:
            sink(FailedEvent(req.request_id, PublicErrorCode.INVALID_REQUEST, False))
            return
        if req.context_ceiling is not None and len(prompt) > req.context_ceiling - req.max_new_tokens:
            # a text prompt is measured against the ceiling once it is tokenized
            sink(FailedEvent(req.request_id, PublicErrorCode.INVALID_REQUEST, False))
            return
        fields = {**req.__dict__, "input_tokens": tuple(prompt), "input_text": None}
        if req.deadline_millis is not None:
            left = receipt + req.deadline_millis / 1000.0 - self.clock()
            if left <= 0.0:
                sink(FailedEvent(req.request_id, PublicErrorCode.DEADLINE_EXCEEDED, False))
                return
            fields["deadline_millis"] = left * 1000.0      # what is left of it, for the scheduler
        try:
            self.engine.submit(GenerateRequest(**fields))
        except AdmissionRejected as e:
            sink(FailedEvent(req.request_id, e.code, e.code is PublicErrorCode.OVERLOADED))
            return
        ctx = req.context_ceiling or self.engine.opts.max_context
        sink(AcceptedWire(req.request_id, req.max_new_tokens, ctx, self.content_digest, self.plan_digest))
        self._live[req.request_id] = _Live(req, sink, IncrementalOutput(req.stop.strings), len(prompt))

    def _on_outputs(self, outs):
        for o in outs:
            lv = self._live.get(o.rid)
            if lv is None:
                continue
            lv.n_out += 1
            delta = b""
            stop_hit = False
            # special tokens (EOS, chat markers) carry no text in the stream,
            # and a string stop never matches inside one
            tok = self.tokenizer
            if tok is not None and o.token in tok.id_to_token and o.token not in tok.added_ids:
                delta, stop_hit = lv.out.push(tok.token_bytes(o.token))
            lv.sink(TokenEvent(o.rid, o.position, o.token, delta))
            if stop_hit and not o.finished:
                self.engine.scheduler.cancel(o.rid)
                self._finish(o.rid, FinishReason.STOP_SEQUENCE)
            elif o.finished:
                self._finish(o.rid, o.reason)

    def _finish(self, rid: int, reason: Optional[FinishReason], error: Optional[PublicErrorCode] = None):
        lv = self._live.pop(rid, None)
        if lv is None:
            return
        res = self.engine.results.get(rid)
        cached = res.cached_tokens if res is not None else 0
        usage = Usage(lv.prompt_len, min(cached, lv.prompt_len), lv.n_out)
        lv.sink(usage)
        if error is not None:
            lv.sink(FailedEvent(rid, error, error in (PublicErrorCode.WORKER_UNAVAILABLE, PublicErrorCode.OVERLOADED)))
        else:
            lv.sink(CompletedEvent(rid, reason or FinishReason.TOKEN_LIMIT, usage, lv.out.finish()))

    def _drain_terminals(self):
        for rid, res in list(self.engine.results.items()):
            if rid in self._live:
                if res.error is not None:
                    self._finish(rid, None, res.error)
                else:
                    self._finish(rid, res.reason)
            self.engine.results.pop(rid, None)

    def _run(self):
        while True:
            with self._cv:
                while not self._inbox and not self.engine.has_work() and not self._stop:
                    self._cv.wait(timeout=0.5)
                if self._stop:
                    break
                items = list(self._inbox)
                self._inbox.clear()
            for kind, a, b in items:
                if kind == "add":
                    try:
                        self._admit(a[0], a[1], b)
                    except Exception:
                        # an admission that fails unexpectedly fails its request,
                        # not the engine loop
                        self._live.pop(a[0].request_id, None)
                        b(FailedEvent(a[0].request_id, PublicErrorCode.INTERNAL, False))
                elif kind == "cancel":
                    self.engine.cancel(a)
                elif kind == "drain_deadline":
                    for rid in list(self._live):
                        self._finish(rid, None, PublicErrorCode.WORKER_UNAVAILABLE)
                        self.engine.cancel(rid)
                    self.engine.results.clear()
                    a.set()
            if self.engine.has_work():
                try:
                    self.engine.step()
                except Exception:
                    self.failed = True
                    self.engine.scheduler.fail_active(PublicErrorCode.WORKER_UNAVAILABLE)
                    self.engine._drain_terminals()
            elif hasattr(self.engine, "idle"):
                # a tensor-parallel leader keeps its followers in lock step while idle
                self.engine.idle()
            self._drain_terminals()


class TCPServer:
    """Framed request-v1 / event-v2 endpoint on asyncio; many concurrent clients."""

    def __init__(self, service: EngineService, host: str = "127.0.0.1", port: int = 0, max_frame: int = 16 << 20,
                 max_pending_events: int = 1 << 16, receipt_timeout_s: float = 30.0, max_connections: int = 4096):
        self.service = service
        # connections beyond this are closed at accept (each holds a frame
        # buffer and an event queue)
        self.max_connections = max_connections
        self.connections = 0
        self.refused_connections = 0
        self.host = host
        self.port = port
        self.max_frame = max_frame
        # A client that stops reading cannot grow the server's memory: past
        # this many undelivered events its requests are cancelled and the
        # connection is closed.
        self.max_pending_events = max_pending_events
        # A frame whose first byte arrived must be complete within this time;
        # a client that stalls mid-frame is disconnected (its partial frame
        # would otherwise hold up to max_frame bytes for as long as it likes).
        self.receipt_timeout_s = receipt_timeout_s
        self.receipt_timeouts = 0
        self.overflows = 0
        self.server: Optional[asyncio.AbstractServer] = None

    async def start(self):
        self.server = await asyncio.start_server(self._client, self.host, self.port)
        self.port = self.server.sockets[0].getsockname()[1]
        return self.port

    async def _client(self, reader: asyncio.StreamReader, writer: asyncio.StreamWriter):
        if self.connections >= self.max_connections:
            self.refused_connections += 1
            writer.close()
            return
        self.connections += 1
        try:
            await self._serve_client(reader, writer)
        finally:
            self.connections -= 1

    async def _serve_client(self, reader: asyncio.StreamReader, writer: asyncio.StreamWriter):
        loop = asyncio.get_running_loop()
        frames = FrameReader(REQUEST_MAGIC, self.max_frame)
        open_rids = set()
        q: asyncio.Queue = asyncio.Queue(maxsize=self.max_pending_events)
        overflow = {"hit": False}

        def put(item):
            if overflow["hit"]:
                return
            try:
                q.put_nowait(item)
            except asyncio.QueueFull:
                overflow["hit"] = True
                self.overflows += 1
                for rid in list(open_rids):
                    self.service.cancel(rid)
                writer.close()

        def sink_for(rid):
            def sink(ev):
                loop.call_soon_threadsafe(put, (rid, ev))
            return sink

        state = {"eof": False}
        done = asyncio.Event()

        async def pump():
            # Writes events in order; a broken transport cancels the client's requests.
            try:
                broken = set()
                while True:
                    rid, ev = await q.get()
                    if ev is not None and rid not in broken:
                        try:
                            frame = encode_event(ev)
                        except FramedWireError:
                            # an event that breaks the stream contract is a server
                            # fault: the request ends with a typed failure
                            broken.add(rid)
                            self.service.cancel(rid)
                            ev = FailedEvent(rid, PublicErrorCode.INTERNAL, False)
                            frame = encode_event(ev)
                        writer.write(frame)
                        await writer.drain()
                        if isinstance(ev, (CompletedEvent, FailedEvent)):
                            open_rids.discard(rid)
                    if state["eof"] and not open_rids:
                        return
            except (ConnectionError, OSError):
                for rid in list(open_rids):
                    self.service.cancel(rid)
            finally:
                done.set()

        pump_task = asyncio.create_task(pump())
        try:
            while True:
                if frames.buf:
                    left = frames.first_byte_time + self.receipt_timeout_s - self.service.clock()
                    try:
                        data = await asyncio.wait_for(reader.read(65536), max(left, 0.0))
                    except asyncio.TimeoutError:
                        self.receipt_timeouts += 1
                        for rid in list(open_rids):
                            self.service.cancel(rid)
                        open_rids.clear()
                        break
                else:
                    data = await reader.read(65536)
                if not data:
                    break
                try:
                    for fr, receipt in frames.feed_timed(data, self.service.clock()):
                        req = decode_request(fr, self.service.limits)
                        if req.request_id in open_rids:
                            raise FramedWireError("request", "duplicate_id")
                        open_rids.add(req.request_id)
                        self.service.submit(req, sink_for(req.request_id), receipt)
                except FramedWireError:
                    # malformed input: drop the connection and its requests
                    for rid in list(open_rids):
                        self.service.cancel(rid)
                    open_rids.clear()
                    break
        finally:
            # A half-closed client still receives the events of its requests.
            state["eof"] = True
            await q.put((0, None))
            await done.wait()
            writer.close()

    async def serve_forever(self):
        async with self.server:
            await self.server.serve_forever()

    def close(self):
        if self.server is not None:
            self.server.close()


class MetricsServer:
    """Minimal HTTP endpoint for the engine's metrics: ``GET /metrics``
    (Prometheus text) and ``GET /health`` (200 while the engine loop runs
    and the service is not draining, 503 otherwise).  Read-only, no request payloads, one response per
    connection."""

    def __init__(self, service: EngineService, host: str = "127.0.0.1", port: int = 0):
        self.service = service
        self.host = host
        self.port = port
        self.server: Optional[asyncio.AbstractServer] = None

    async def start(self):
        self.server = await asyncio.start_server(self._client, self.host, self.port)
        self.port = self.server.sockets[0].getsockname()[1]
        return self.port

    async def _client(self, reader: asyncio.StreamReader, writer: asyncio.StreamWriter):
        try:
            line = await asyncio.wait_for(reader.readline(), 5.0)
            parts = line.decode("latin-1").split()
            path = parts[1] if len(parts) >= 2 and parts[0] == "GET" else ""
            if path == "/metrics":
                body = self.service.engine.metrics.registry.render_prometheus().encode()
                status = "200 OK"
            elif path == "/health":
                alive = self.service.alive() and not self.service.draining
                body = b"ok\n" if alive else (b"draining\n" if self.service.draining else b"unavailable\n")
                status = "200 OK" if alive else "503 Service Unavailable"
            else:
                body, status = b"not found\n", "404 Not Found"
            writer.write(f"HTTP/1.1 {status}\r\nContent-Type: text/plain; version=0.0.4\r\n"
                         f"Content-Length: {len(body)}\r\nConnection: close\r\n\r\n".encode() + body)
            await writer.drain()
        except (asyncio.TimeoutError, ConnectionError, OSError):
            pass
        finally:
            writer.close()

    async def stop(self):
        if self.server is not None:
            self.server.close()
            await self.server.wait_closed()
