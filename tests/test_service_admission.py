"""Request admission in the serving layer (CPU): receipt times, deadlines,
model identity, token and text checks, string stops, cancellation and worker
failure, each seen as the event stream a client receives.

Modelled on the reference's service/request_admission tests
(request_admission_test.mbt: "public framed receipt and Luna preparation use
the monotonic clock", "identity receipt and expired budget reject before
publication", "text admission preserves receipt deadline and separates string
stops", "string stops remain in incremental output instead of scheduler
state", "deadline samples once before and once after tokenization",
"direct framed preparation is equivalent across every chunk size") and
service/online_session (Accepted -> Token* -> Usage -> Completed | Failed).
"""
import threading
import time

import pytest

from lunaflux_b200.config import CacheConfig, SchedulerConfig
from lunaflux_b200.contracts.inference import (CompletedEvent, FailedEvent, FinishReason, GenerateRequest,
                                               PublicErrorCode, StopConditions, TokenEvent, Usage, default_limits)
from lunaflux_b200.engine.engine import EngineOptions, LLMEngine
from lunaflux_b200.models.spec import tiny_llama
from lunaflux_b200.models.weights import build_runtime, random_checkpoint
from lunaflux_b200.oracle.reference import ReferenceModel
from lunaflux_b200.runtime.clock import FakeClock
from lunaflux_b200.service.framed_wire import REQUEST_MAGIC, AcceptedWire, FrameReader, encode_request
from lunaflux_b200.service.server import EngineService
from lunaflux_b200.testing.fake_device import FaultPlan, FakeDeviceOps
from lunaflux_b200.tokenizer.bpe import synthetic_byte_tokenizer

LIM = default_limits(256, 512)


@pytest.fixture(scope="module")
def tiny():
    spec = tiny_llama()
    return spec, random_checkpoint(spec, 0)


class Client:
    """Collects each request's events; waits for its terminal event."""

    def __init__(self):
        self.events = {}
        self.lock = threading.Lock()
        self.cv = threading.Condition(self.lock)

    def sink(self, rid):
        def f(ev):
            with self.cv:
                self.events.setdefault(rid, []).append(ev)
                self.cv.notify_all()
        return f

    def wait(self, rid, timeout=60.0):
        end = time.monotonic() + timeout
        with self.cv:
            while True:
                evs = self.events.get(rid, [])
                if evs and isinstance(evs[-1], (CompletedEvent, FailedEvent)):
                    return list(evs)
                left = end - time.monotonic()
                assert left > 0, f"request {rid} did not finish: {evs}"
                self.cv.wait(left)


def service(tiny, ops=None, tokenizer=None, clock=None, **kw):
    spec, ck = tiny
    eng = LLMEngine(build_runtime(spec, lambda n: ck[n]), ops or FakeDeviceOps(), "cpu",
                    SchedulerConfig(step_token_budget=64, max_active_requests=4, prefill_chunk_tokens=64,
                                    emergency_decode_page_reserve=1),
                    CacheConfig(), EngineOptions(max_context=256, num_pages=64, graph_sizes=()))
    svc = EngineService(eng, tokenizer, LIM, content_digest=kw.pop("content_digest", ""),
                        clock=clock or time.monotonic, **kw)
    return svc, eng


def terminal(evs):
    return evs[-1]


# ----------------------------------------------------------------------------- event order
def test_event_order_accepted_tokens_usage_completed(tiny):
    spec, ck = tiny
    svc, _ = service(tiny)
    c = Client()
    svc.start()
    try:
        svc.submit(GenerateRequest(1, input_tokens=(5, 6, 7), max_new_tokens=5), c.sink(1))
        evs = c.wait(1)
    finally:
        svc.stop()
    assert isinstance(evs[0], AcceptedWire)
    toks = [e for e in evs if isinstance(e, TokenEvent)]
    assert [e.token_id for e in toks] == ReferenceModel(spec, ck).generate_greedy([5, 6, 7], 5)
    assert [e.position for e in toks] == [3, 4, 5, 6, 7]
    assert isinstance(evs[-2], Usage) and (evs[-2].input_tokens, evs[-2].output_tokens) == (3, 5)
    assert isinstance(evs[-1], CompletedEvent) and evs[-1].reason is FinishReason.TOKEN_LIMIT
    assert len(evs) == 1 + 5 + 2


# ----------------------------------------------------------------------------- identity and inputs
@pytest.mark.parametrize("field", ["model_content_digest", "model_plan_digest"])
def test_wrong_model_identity_fails_before_the_engine_sees_it(tiny, field):
    svc, eng = service(tiny, content_digest="c" * 64)
    c = Client()
    svc.start()
    try:
        svc.submit(GenerateRequest(1, input_tokens=(5,), max_new_tokens=2, **{field: "0" * 64}), c.sink(1))
        evs = c.wait(1)
        ok = {"model_content_digest": "c" * 64, "model_plan_digest": svc.plan_digest}[field]
        svc.submit(GenerateRequest(2, input_tokens=(5,), max_new_tokens=2, **{field: ok}), c.sink(2))
        good = c.wait(2)
    finally:
        svc.stop()
    assert evs == [FailedEvent(1, PublicErrorCode.INVALID_REQUEST, False)]
    assert isinstance(good[-1], CompletedEvent)
    assert eng.metrics.requests.get() == 1


def test_token_ids_and_context_ceiling_are_checked_against_the_loaded_model(tiny):
    svc, eng = service(tiny)
    c = Client()
    svc.start()
    try:
        svc.submit(GenerateRequest(1, input_tokens=(5, 256), max_new_tokens=2), c.sink(1))      # vocab is 256
        svc.submit(GenerateRequest(2, input_tokens=(5, 6, 7), max_new_tokens=8, context_ceiling=10), c.sink(2))
        svc.submit(GenerateRequest(3, input_text=b"abc", max_new_tokens=2), c.sink(3))         # no tokenizer
        evs = [c.wait(r) for r in (1, 2, 3)]
    finally:
        svc.stop()
    for rid, e in zip((1, 2, 3), evs):
        assert e == [FailedEvent(rid, PublicErrorCode.INVALID_REQUEST, False)], (rid, e)
    assert eng.metrics.requests.get() == 0


def test_text_admission_tokenizes_off_the_engine_thread_and_keeps_string_stops_out_of_the_scheduler(tiny):
    """A string stop lives in the incremental output: the scheduler gets only
    token stops, and the text is cut before the stop string."""
    spec, ck = tiny
    tok = synthetic_byte_tokenizer()
    prompt = tok.encode("hello")
    want = ReferenceModel(spec, ck).generate_greedy(prompt, 12)
    text = b"".join(tok.token_bytes(t) for t in want)
    stop = text[3:5]                       # bytes the 4th and 5th tokens produce
    assert stop not in text[:4]
    svc, eng = service(tiny, tokenizer=tok)
    seen = []
    orig = eng.submit
    eng.submit = lambda g: (seen.append(g), orig(g))[1]
    c = Client()
    svc.start()
    try:
        svc.submit(GenerateRequest(1, input_text=b"hello", max_new_tokens=12, stop=StopConditions((), (stop,))),
                   c.sink(1))
        evs = c.wait(1)
    finally:
        svc.stop()
    (g,) = seen
    assert g.input_tokens == tuple(prompt) and g.input_text is None and g.stop.token_ids == ()
    done = evs[-1]
    assert isinstance(done, CompletedEvent) and done.reason is FinishReason.STOP_SEQUENCE
    # stops match the raw bytes; what is delivered is valid UTF-8 (U+FFFD for bad bytes)
    delivered = b"".join(e.delta for e in evs if isinstance(e, TokenEvent)) + done.final_delta
    assert delivered == text[:text.index(stop)].decode("utf-8", "replace").encode("utf-8")
    assert not eng.has_work()              # the engine request was cancelled at the stop


# ----------------------------------------------------------------------------- deadlines
def test_expired_receipt_budget_rejects_before_publication(tiny):
    clock = FakeClock()
    svc, eng = service(tiny, clock=clock)
    c = Client()
    svc.start()
    try:
        receipt = clock()
        clock.advance(0.25)
        svc.submit(GenerateRequest(1, input_tokens=(5,), max_new_tokens=2, deadline_millis=250), c.sink(1), receipt)
        evs = c.wait(1)
    finally:
        svc.stop()
    assert evs == [FailedEvent(1, PublicErrorCode.DEADLINE_EXCEEDED, False)]
    assert eng.metrics.requests.get() == 0


def test_the_scheduler_gets_what_is_left_of_the_deadline(tiny):
    clock = FakeClock()
    svc, eng = service(tiny, clock=clock)
    seen = []
    orig = eng.submit
    eng.submit = lambda g: (seen.append(g), orig(g))[1]
    c = Client()
    svc.start()
    try:
        receipt = clock()
        clock.advance(0.4)                         # the request spent 400 ms reaching the service
        svc.submit(GenerateRequest(1, input_tokens=(5,), max_new_tokens=2, deadline_millis=1000), c.sink(1), receipt)
        c.wait(1)
    finally:
        svc.stop()
    (g,) = seen
    assert g.deadline_millis == pytest.approx(600.0)


def test_deadline_is_checked_again_after_tokenization(tiny):
    clock = FakeClock()
    tok = synthetic_byte_tokenizer()

    class SlowTokenizer:
        def __getattr__(self, name):
            return getattr(tok, name)

        def encode_bytes(self, data, allow_special=True):
            clock.advance(1.0)                     # tokenization outlasts the deadline
            return tok.encode_bytes(data, allow_special)

    svc, eng = service(tiny, tokenizer=SlowTokenizer(), clock=clock)
    c = Client()
    svc.start()
    try:
        svc.submit(GenerateRequest(1, input_text=b"abc", max_new_tokens=2, deadline_millis=500), c.sink(1))
        evs = c.wait(1)
    finally:
        svc.stop()
    assert evs == [FailedEvent(1, PublicErrorCode.DEADLINE_EXCEEDED, False)]
    assert eng.metrics.requests.get() == 0


@pytest.mark.parametrize("chunk", [1, 7, 16, 64, 1000])
def test_frame_receipt_is_the_arrival_of_its_first_byte(chunk):
    frames = [encode_request(GenerateRequest(r, input_tokens=tuple(range(1, 3 + r)), max_new_tokens=2))
              for r in (1, 2, 3)]
    stream = b"".join(frames)
    starts = [sum(len(f) for f in frames[:i]) for i in range(3)]
    reader = FrameReader(REQUEST_MAGIC)
    got = []
    for k, off in enumerate(range(0, len(stream), chunk)):
        for f, t in reader.feed_timed(stream[off:off + chunk], float(k)):
            got.append((f, t))
    assert [f for f, _ in got] == frames
    # the receipt is the index of the chunk that held the frame's first byte
    assert [t for _, t in got] == [float(s // chunk) for s in starts]


# ----------------------------------------------------------------------------- cancel and failure
def test_cancel_mid_stream_ends_with_a_cancelled_completion(tiny):
    svc, eng = service(tiny)
    c = Client()
    svc.start()
    try:
        svc.submit(GenerateRequest(1, input_tokens=(5, 6), max_new_tokens=200), c.sink(1))
        end = time.monotonic() + 30
        while not any(isinstance(e, TokenEvent) for e in c.events.get(1, [])):
            assert time.monotonic() < end
            time.sleep(0.002)
        svc.cancel(1)
        evs = c.wait(1)
    finally:
        svc.stop()
    assert isinstance(evs[-1], CompletedEvent) and evs[-1].reason is FinishReason.CANCELLED
    assert sum(isinstance(e, TokenEvent) for e in evs) < 200
    assert not eng.has_work()
    eng.scheduler.debug_check_invariants()
    assert eng.scheduler.allocator.free_page_count() == eng.scheduler.allocator.capacity


def test_a_failed_step_fails_active_requests_retryably_and_later_ones_too(tiny):
    svc, eng = service(tiny, ops=FakeDeviceOps(FaultPlan(at_forward=3, kind="launch_error")))
    c = Client()
    svc.start()
    try:
        svc.submit(GenerateRequest(1, input_tokens=(5, 6), max_new_tokens=50), c.sink(1))
        first = c.wait(1)
        svc.submit(GenerateRequest(2, input_tokens=(5, 6), max_new_tokens=2), c.sink(2))
        later = c.wait(2)
    finally:
        svc.stop()
    assert first[-1] == FailedEvent(1, PublicErrorCode.WORKER_UNAVAILABLE, True)
    assert [e.position for e in first if isinstance(e, TokenEvent)] == [2, 3]
    assert later == [FailedEvent(2, PublicErrorCode.WORKER_UNAVAILABLE, True)]
    assert not svc.alive()


def test_an_unexpected_admission_error_fails_only_its_request(tiny):
    svc, eng = service(tiny)
    orig = eng.submit

    def flaky(g):
        if g.request_id == 1:
            raise RuntimeError("backend refused the request")
        return orig(g)

    eng.submit = flaky
    c = Client()
    svc.start()
    try:
        svc.submit(GenerateRequest(1, input_tokens=(5, 6), max_new_tokens=2), c.sink(1))
        first = c.wait(1)
        svc.submit(GenerateRequest(2, input_tokens=(5, 6), max_new_tokens=2), c.sink(2))
        second = c.wait(2)
    finally:
        svc.stop()
    assert first == [FailedEvent(1, PublicErrorCode.INTERNAL, False)]
    assert isinstance(second[-1], CompletedEvent)


def test_a_client_stalled_mid_frame_is_disconnected(tiny):
    """A frame must be complete within the receipt timeout of its first byte
    (reference: request_admission 'pre-View hard receipt deadline expires and
    frees scanner authority'); a connection that only sent whole frames is not
    affected by the timeout."""
    import asyncio
    from lunaflux_b200.service.server import TCPServer
    svc, _ = service(tiny)
    svc.start()
    frame = encode_request(GenerateRequest(1, input_tokens=(5, 6), max_new_tokens=2))

    async def main():
        server = TCPServer(svc, receipt_timeout_s=0.3)
        port = await server.start()
        # an idle connection with no partial frame stays open
        r0, w0 = await asyncio.open_connection("127.0.0.1", port)
        r, w = await asyncio.open_connection("127.0.0.1", port)
        w.write(frame[:40])
        await w.drain()
        t0 = time.monotonic()
        rest = await asyncio.wait_for(r.read(), 10)          # EOF once the server drops us
        waited = time.monotonic() - t0
        idle_open = not r0.at_eof()
        w.close()
        w0.close()
        server.close()
        return rest, waited, server.receipt_timeouts, idle_open

    try:
        rest, waited, n, idle_open = asyncio.run(main())
    finally:
        svc.stop()
    assert rest == b"" and 0.2 <= waited < 5.0 and n == 1 and idle_open


def test_connections_beyond_the_limit_are_closed_at_accept(tiny):
    import asyncio
    from lunaflux_b200.service.server import TCPServer
    svc, _ = service(tiny)
    svc.start()

    async def main():
        server = TCPServer(svc, max_connections=2)
        port = await server.start()
        conns = [await asyncio.open_connection("127.0.0.1", port) for _ in range(2)]
        await asyncio.sleep(0.2)
        r3, w3 = await asyncio.open_connection("127.0.0.1", port)
        third = await asyncio.wait_for(r3.read(), 5)         # closed by the server
        for _, w in conns:
            w.close()
        w3.close()
        await asyncio.sleep(0.2)
        # a slot freed by a closed connection is usable again
        r4, w4 = await asyncio.open_connection("127.0.0.1", port)
        w4.write(encode_request(GenerateRequest(4, input_tokens=(5, 6), max_new_tokens=1)))
        await w4.drain()
        got = await asyncio.wait_for(r4.read(208), 10)
        w4.close()
        server.close()
        return third, got, server.refused_connections

    try:
        third, got, refused = asyncio.run(main())
    finally:
        svc.stop()
    assert third == b"" and refused == 1 and len(got) > 0


def test_a_failing_sink_does_not_end_the_engine_thread(tiny):
    svc, _ = service(tiny)
    c = Client()

    def broken(ev):
        raise RuntimeError("Event loop is closed")

    svc.start()
    try:
        svc.submit(GenerateRequest(1, input_tokens=(5, 6), max_new_tokens=3), broken)
        svc.submit(GenerateRequest(2, input_tokens=(5, 6), max_new_tokens=3), c.sink(2))
        evs = c.wait(2)
        assert svc.alive()
    finally:
        svc.stop()
    assert isinstance(evs[-1], CompletedEvent)


def test_special_tokens_carry_no_text_in_the_stream():
    """Generated special tokens (EOS, chat markers) are streamed as token ids
    with an empty delta, so no "<|eot_id|>" text reaches the client
    (reference: service/incremental_output/output_wbtest.mbt, skipped
    specials are payload safe)."""
    from lunaflux_b200.models.spec import LlamaSpec
    from lunaflux_b200.tokenizer.bpe import Tokenizer, byte_alphabet
    spec = LlamaSpec(hidden=64, layers=2, heads=4, kv_heads=2, head_dim=16, ffn=172, vocab=512, rope_theta=10000.0,
                     max_position=512, dtype="fp32")
    ck = random_checkpoint(spec, 0)
    alpha = byte_alphabet()
    tok = Tokenizer({alpha[b]: b for b in range(256)}, [], [(f"<|s{i}|>", i) for i in range(256, 512)])
    prompt = tok.encode("hello")
    want = ReferenceModel(spec, ck).generate_greedy(prompt, 24)
    assert any(t >= 256 for t in want) and any(t < 256 for t in want)   # both kinds are generated
    svc, eng = service((spec, ck), tokenizer=tok)
    c = Client()
    svc.start()
    try:
        svc.submit(GenerateRequest(1, input_text=b"hello", max_new_tokens=24), c.sink(1))
        evs = c.wait(1)
    finally:
        svc.stop()
    toks = [e for e in evs if isinstance(e, TokenEvent)]
    assert [e.token_id for e in toks] == want
    assert all(e.delta == b"" for e in toks if e.token_id >= 256)
    delivered = b"".join(e.delta for e in toks) + evs[-1].final_delta
    text = b"".join(bytes([t]) for t in want if t < 256)
    assert delivered == text.decode("utf-8", "replace").encode("utf-8")
