"""Framed wire codecs, incremental output and the TCP serving path (CPU)."""
import asyncio
import struct

import pytest
import torch

from lunaflux_b200.contracts.inference import (CachePermission, CacheScope, CompletedEvent, FailedEvent,
                                               FinishReason, GenerateRequest, PublicErrorCode, SamplingParameters,
                                               StopConditions, TokenEvent, Usage, default_limits)
from lunaflux_b200.service.detokenize import IncrementalOutput
from lunaflux_b200.service.framed_wire import (EVENT_MAGIC, AcceptedWire, FrameReader, FramedWireError, decode_event,
                                               decode_request, encode_event, encode_request, fnv1a)

LIM = default_limits(256, 512)


def full_request():
    return GenerateRequest(request_id=77, input_tokens=(1, 2, 3, 250), max_new_tokens=9, context_ceiling=300,
                           sampling=SamplingParameters.sample(0.7, top_k=40, top_p=0.9, seed=5),
                           stop=StopConditions((7, 9), (b"ab", b"\xc3\xa9")), streaming=True, deadline_millis=1500,
                           cache=CacheScope(b"tenant-1", CachePermission.READ_ONLY), trace=b"trace:1",
                           model_plan_digest="a" * 64)


def test_request_layout_offsets():
    fr = encode_request(full_request())
    magic, ver, kind, total = struct.unpack_from("<IIII", fr, 0)
    assert (magic, ver, kind, total) == (0x5152464C, 1, 1, len(fr))
    assert struct.unpack_from("<I", fr, 20)[0] == 2 | 4 | 8 | 16 | 32
    assert struct.unpack_from("<i", fr, 28)[0] == 4 and struct.unpack_from("<i", fr, 52)[0] == 9
    assert struct.unpack_from("<d", fr, 72)[0] == 0.7 and struct.unpack_from("<Q", fr, 104)[0] == 77
    assert fr[176:240] == b"a" * 64 and struct.unpack_from("<i", fr, 240)[0] == 1
    assert struct.unpack_from("<i", fr, 248)[0] == 256
    assert struct.unpack_from("<I", fr, 16)[0] == fnv1a(fr)


def test_request_roundtrip():
    req = full_request()
    assert decode_request(encode_request(req), LIM) == req.validate(LIM)
    t = GenerateRequest(request_id=1, input_text="héllo".encode(), max_new_tokens=2)
    assert decode_request(encode_request(t), LIM) == t


@pytest.mark.parametrize("mutate,rule", [
    (lambda b: b.__setitem__(slice(0, 4), b"XXXX"), "magic"),
    (lambda b: b.__setitem__(300, b[300] ^ 1), "checksum"),
    (lambda b: b.__setitem__(slice(4, 8), struct.pack("<I", 2)), "version"),
])
def test_request_hostile(mutate, rule):
    b = bytearray(encode_request(full_request()))
    mutate(b)
    with pytest.raises(FramedWireError) as e:
        decode_request(bytes(b), LIM)
    assert e.value.rule == rule


def _fix_checksum(b):
    struct.pack_into("<I", b, 16, fnv1a(b))
    return bytes(b)


def test_request_nonzero_reserved_and_unused_rejected():
    b = bytearray(encode_request(GenerateRequest(1, input_tokens=(1,), max_new_tokens=1)))
    b[253] = 1
    with pytest.raises(FramedWireError):
        decode_request(_fix_checksum(b), LIM)
    b = bytearray(encode_request(GenerateRequest(1, input_tokens=(1,), max_new_tokens=1)))
    struct.pack_into("<i", b, 64, 5)  # top_k without its flag
    with pytest.raises(FramedWireError):
        decode_request(_fix_checksum(b), LIM)
    with pytest.raises(FramedWireError):
        decode_request(encode_request(GenerateRequest(1, input_tokens=(999,), max_new_tokens=1)), LIM)


def test_event_roundtrip_and_layout():
    evs = [AcceptedWire(3, 9, 300, "", "b" * 64), TokenEvent(3, 12, 99, "é".encode()), TokenEvent(3, 13, 5, b""),
           Usage(4, 0, 2), CompletedEvent(3, FinishReason.STOP_SEQUENCE, Usage(4, 2, 2), b"tail"),
           FailedEvent(3, PublicErrorCode.WORKER_UNAVAILABLE, True)]
    for ev in evs:
        fr = encode_event(ev)
        assert struct.unpack_from("<II", fr, 0) == (EVENT_MAGIC, 2)
        assert struct.unpack_from("<i", fr, 196)[0] == 208
        back = decode_event(fr, 3)
        assert back == ev
    fr = encode_event(TokenEvent(3, 12, 99, b"x"))
    assert struct.unpack_from("<ii", fr, 24) == (99, 12) and struct.unpack_from("<I", fr, 20)[0] == 1
    fr = encode_event(CompletedEvent(3, FinishReason.CANCELLED, Usage(4, 0, 1)))
    assert struct.unpack_from("<i", fr, 24)[0] == 2 and struct.unpack_from("<iiii", fr, 32) == (4, 0, 1, 5)
    assert decode_event(encode_event(FailedEvent(1, PublicErrorCode.DEADLINE_EXCEEDED, False)), 1).code \
        is PublicErrorCode.DEADLINE_EXCEEDED


def test_frame_reader_splits_and_poisons():
    a = encode_event(Usage(1, 0, 1))
    b = encode_event(Usage(2, 0, 3))
    r = FrameReader(EVENT_MAGIC, header=208)
    assert r.feed(a[:10]) == []
    assert r.feed(a[10:] + b[:100]) == [a]
    assert r.feed(b[100:]) == [b]
    with pytest.raises(FramedWireError):
        r.feed(b"\x00" * 16)


def test_frame_reader_is_chunk_size_invariant():
    """Three request frames fed in chunks of every size from 1 byte to the
    whole stream come out as the same frames and decode to the same requests
    (reference: service/request_admission, 'direct framed preparation is
    equivalent across every chunk size')."""
    from lunaflux_b200.service.framed_wire import REQUEST_MAGIC
    reqs = [full_request(), GenerateRequest(request_id=5, input_tokens=(3,), max_new_tokens=1),
            GenerateRequest(request_id=6, input_tokens=tuple(range(40)), max_new_tokens=4,
                            stop=StopConditions((), (b"x",)))]
    frames = [encode_request(r) for r in reqs]
    stream = b"".join(frames)
    for chunk in range(1, len(stream) + 1):
        rd = FrameReader(REQUEST_MAGIC)
        got = []
        for o in range(0, len(stream), chunk):
            got += rd.feed(stream[o:o + chunk])
        assert got == frames, chunk
        assert [decode_request(f, LIM) for f in got] == reqs
        assert not rd.buf


def test_incremental_output_stop_across_tokens_and_utf8():
    o = IncrementalOutput([b"STOP"])
    assert o.push(b"hello S") == (b"hello ", False)  # "S" withheld: may start STOP
    assert o.push(b"T") == (b"", False)
    assert o.push(b"Xy") == (b"STXy", False)
    assert o.push(b"zzST") == (b"zz", False)
    assert o.push(b"OPmore") == (b"", True)
    o = IncrementalOutput()
    e = "é".encode()
    assert o.push(e[:1]) == (b"", False)  # incomplete code point withheld
    assert o.push(e[1:] + b"!") == (e + b"!", False)
    assert o.push(b"\xf0\x9f") == (b"", False)
    assert o.finish() == "�".encode()


def test_tcp_end_to_end():
    from lunaflux_b200.config import CacheConfig, SchedulerConfig
    from lunaflux_b200.engine.engine import EngineOptions, LLMEngine
    from lunaflux_b200.models.spec import tiny_llama
    from lunaflux_b200.models.weights import build_runtime, random_checkpoint
    from lunaflux_b200.ops.torch_ops import TorchOps
    from lunaflux_b200.oracle.reference import ReferenceModel
    from lunaflux_b200.service.framed_wire import EVENT_HEADER
    from lunaflux_b200.service.server import EngineService, MetricsServer, TCPServer
    from lunaflux_b200.tokenizer.bpe import synthetic_byte_tokenizer

    spec = tiny_llama()
    ck = random_checkpoint(spec, 0)
    eng = LLMEngine(build_runtime(spec, lambda n: ck[n]), TorchOps(), "cpu",
                    SchedulerConfig(step_token_budget=64, max_active_requests=4, prefill_chunk_tokens=64,
                                    emergency_decode_page_reserve=1),
                    CacheConfig(), EngineOptions(max_context=256, num_pages=64, graph_sizes=()))
    svc = EngineService(eng, synthetic_byte_tokenizer(), LIM)
    svc.start()
    prompt = [5, 17, 99, 3, 200]
    expect = ReferenceModel(spec, ck).generate_greedy(prompt, 6)

    async def client(req):
        r, w = await asyncio.open_connection("127.0.0.1", port)
        w.write(encode_request(req))
        await w.drain()
        fr = FrameReader(EVENT_MAGIC, header=EVENT_HEADER)
        events = []
        while True:
            data = await r.read(65536)
            if not data:
                break
            for f in fr.feed(data):
                events.append(decode_event(f, req.request_id))
            if events and isinstance(events[-1], (CompletedEvent, FailedEvent)):
                break
        w.close()
        return events

    async def main():
        global port
        server = TCPServer(svc)
        p = await server.start()
        globals()["port"] = p
        a, b, c = await asyncio.gather(
            client(GenerateRequest(1, input_tokens=tuple(prompt), max_new_tokens=6)),
            client(GenerateRequest(2, input_text=b"hi there", max_new_tokens=4)),
            client(GenerateRequest(3, input_tokens=(1,), max_new_tokens=4, model_plan_digest="f" * 64)))
        server.close()
        # the metrics endpoint: Prometheus text and the health probe
        ms = MetricsServer(svc)
        mp = await ms.start()
        texts = []
        for path in ("/metrics", "/health", "/nope"):
            r, w = await asyncio.open_connection("127.0.0.1", mp)
            w.write(f"GET {path} HTTP/1.1\r\nHost: x\r\n\r\n".encode())
            await w.drain()
            texts.append((await r.read()).decode())
            w.close()
        await ms.stop()
        return a, b, c, texts

    try:
        a, b, c, texts = asyncio.run(main())
    finally:
        svc.stop()
    assert texts[0].startswith("HTTP/1.1 200") and "lunaflux_output_tokens_total" in texts[0]
    assert "lunaflux_ttft_seconds_count 2" in texts[0]
    assert texts[1].startswith("HTTP/1.1 200") and texts[2].startswith("HTTP/1.1 404")
    assert isinstance(a[0], AcceptedWire)
    toks = [e.token_id for e in a if isinstance(e, TokenEvent)]
    assert toks == expect
    assert isinstance(a[-2], Usage) and a[-2].output_tokens == 6
    assert isinstance(a[-1], CompletedEvent) and a[-1].reason is FinishReason.TOKEN_LIMIT
    assert isinstance(b[-1], CompletedEvent) and sum(isinstance(e, TokenEvent) for e in b) == 4
    assert isinstance(c[-1], FailedEvent) and c[-1].code is PublicErrorCode.INVALID_REQUEST


def test_tcp_many_clients_overlapped_with_disconnects():
    """Twelve concurrent TCP clients on an engine with overlapped steps; three
    disconnect after their first token.  Every other client receives the
    oracle's tokens, a usage record and one terminal event; the engine drains
    and every KV page returns."""
    import random
    from lunaflux_b200.config import CacheConfig, SchedulerConfig
    from lunaflux_b200.engine.engine import EngineOptions, LLMEngine
    from lunaflux_b200.models.spec import tiny_llama
    from lunaflux_b200.models.weights import build_runtime, random_checkpoint
    from lunaflux_b200.ops.torch_ops import TorchOps
    from lunaflux_b200.oracle.reference import ReferenceModel
    from lunaflux_b200.service.framed_wire import EVENT_HEADER
    from lunaflux_b200.service.server import EngineService, TCPServer
    from lunaflux_b200.tokenizer.bpe import synthetic_byte_tokenizer

    spec = tiny_llama()
    ck = random_checkpoint(spec, 0)
    ref = ReferenceModel(spec, ck)
    eng = LLMEngine(build_runtime(spec, lambda n: ck[n]), TorchOps(), "cpu",
                    SchedulerConfig(step_token_budget=48, max_active_requests=4, prefill_chunk_tokens=48,
                                    emergency_decode_page_reserve=1),
                    CacheConfig(prefix_enabled=False),
                    EngineOptions(max_context=256, num_pages=24, graph_sizes=(), overlap_steps=True))
    svc = EngineService(eng, synthetic_byte_tokenizer(), LIM)
    svc.start()
    rnd = random.Random(7)
    jobs = [(100 + i, tuple(rnd.randrange(256) for _ in range(rnd.randint(2, 30))), rnd.randint(3, 9), i in (2, 5, 9))
            for i in range(12)]

    async def client(port, rid, prompt, n, drop):
        r, w = await asyncio.open_connection("127.0.0.1", port)
        w.write(encode_request(GenerateRequest(rid, input_tokens=prompt, max_new_tokens=n)))
        await w.drain()
        fr = FrameReader(EVENT_MAGIC, header=EVENT_HEADER)
        events = []
        while True:
            data = await r.read(65536)
            if not data:
                break
            for f in fr.feed(data):
                events.append(decode_event(f, rid))
            if drop and any(isinstance(e, TokenEvent) for e in events):
                break
            if events and isinstance(events[-1], (CompletedEvent, FailedEvent)):
                break
        w.close()
        return events

    async def main():
        server = TCPServer(svc)
        port = await server.start()
        outs = await asyncio.gather(*(client(port, *j) for j in jobs))
        for _ in range(200):                       # the dropped requests are cancelled and drained
            if not eng.has_work() and not eng.live:
                break
            await asyncio.sleep(0.05)
        server.close()
        return outs

    try:
        outs = asyncio.run(main())
    finally:
        svc.stop()
    for (rid, prompt, n, drop), ev in zip(jobs, outs):
        toks = [e.token_id for e in ev if isinstance(e, TokenEvent)]
        if drop:
            assert toks and toks == ref.generate_greedy(list(prompt), n)[:len(toks)]
            continue
        assert toks == ref.generate_greedy(list(prompt), n), rid
        assert isinstance(ev[-2], Usage) and ev[-2].output_tokens == n
        assert isinstance(ev[-1], CompletedEvent)
        assert sum(isinstance(e, (CompletedEvent, FailedEvent)) for e in ev) == 1
    assert not eng.has_work()
    assert eng.scheduler.allocator.allocated_page_count() == 0


def test_request_decoder_fuzz():
    """Random mutations of a valid frame and random bytes: the decoder either
    returns a request that passes validation or raises FramedWireError;
    nothing else escapes."""
    import random
    base = encode_request(full_request())
    rnd = random.Random(5)
    outcomes = {"ok": 0, "rejected": 0}
    for i in range(3000):
        if i % 3 == 0:
            data = bytes(rnd.randrange(256) for _ in range(rnd.randint(0, 200)))
        else:
            b = bytearray(base)
            for _ in range(rnd.randint(1, 6)):
                b[rnd.randrange(len(b))] = rnd.randrange(256)
            if rnd.random() < 0.2:
                b = b[: rnd.randrange(len(b))]
            data = bytes(b)
        try:
            req = decode_request(data, LIM)
            req.validate(LIM)
            outcomes["ok"] += 1
        except FramedWireError:
            outcomes["rejected"] += 1
    assert outcomes["rejected"] > 2000 and outcomes["ok"] >= 0


def test_graceful_drain():
    """drain(): new requests are refused (retryable overloaded), live ones may
    finish until the deadline, the rest fail with the retryable
    worker_unavailable code and are cancelled in the engine."""
    import threading
    import time

    from lunaflux_b200.config import CacheConfig, SchedulerConfig
    from lunaflux_b200.contracts import CompletedEvent, FailedEvent, GenerateRequest, PublicErrorCode
    from lunaflux_b200.engine.engine import EngineOptions, LLMEngine
    from lunaflux_b200.models.spec import tiny_llama
    from lunaflux_b200.models.weights import build_runtime, random_checkpoint
    from lunaflux_b200.ops.torch_ops import TorchOps
    from lunaflux_b200.service.server import EngineService

    spec = tiny_llama()
    ck = random_checkpoint(spec, 0)

    def service():
        eng = LLMEngine(build_runtime(spec, lambda n: ck[n]), TorchOps(), "cpu",
                        SchedulerConfig(step_token_budget=64, max_active_requests=4, prefill_chunk_tokens=64,
                                        emergency_decode_page_reserve=1),
                        CacheConfig(), EngineOptions(max_context=512, num_pages=128, graph_sizes=()))
        svc = EngineService(eng, None, LIM)
        svc.start()
        return svc, eng

    ends = {}
    lock = threading.Lock()

    def sink(rid):
        def f(ev):
            if isinstance(ev, (CompletedEvent, FailedEvent)):
                with lock:
                    ends[rid] = ev
        return f

    # short requests finish inside the drain window
    svc, eng = service()
    for rid in (1, 2):
        svc.submit(GenerateRequest(request_id=rid, input_tokens=(3, 4, 5), max_new_tokens=3), sink(rid))
    assert svc.drain(30.0)
    assert isinstance(ends[1], CompletedEvent) and isinstance(ends[2], CompletedEvent)
    svc.submit(GenerateRequest(request_id=3, input_tokens=(3, 4), max_new_tokens=2), sink(3))
    t0 = time.monotonic()
    while 3 not in ends and time.monotonic() - t0 < 10:
        time.sleep(0.01)
    assert isinstance(ends[3], FailedEvent) and ends[3].code is PublicErrorCode.OVERLOADED and ends[3].retryable
    svc.stop()

    # a long request outlives the deadline: it fails retryably and leaves the engine
    svc, eng = service()
    svc.submit(GenerateRequest(request_id=10, input_tokens=(7, 8, 9), max_new_tokens=400), sink(10))
    t0 = time.monotonic()
    while not eng.has_work() and time.monotonic() - t0 < 10:
        time.sleep(0.005)
    assert not svc.drain(0.05)
    ev = ends[10]
    assert isinstance(ev, FailedEvent) and ev.code is PublicErrorCode.WORKER_UNAVAILABLE and ev.retryable
    t0 = time.monotonic()
    while eng.has_work() and time.monotonic() - t0 < 10:
        time.sleep(0.01)
    assert not eng.has_work()
    svc.stop()


def test_incremental_output_is_payload_safe_and_split_invariant():
    """Random byte pieces (valid text, stray continuation bytes, 0xFF,
    truncated sequences), no stop strings: every delta is valid UTF-8 and the
    deltas plus the terminal tail equal the replacement-decoded whole output,
    however the bytes were split into tokens (reference: incremental_output
    'UTF-8 split across byte tokens publishes only a complete scalar',
    'invalid UTF-8 unknown tokens ... are payload safe')."""
    import random
    rng = random.Random(3)
    alphabet = [b"a", b"\xc3\xa9", b"\xe2\x82\xac", b"\xf0\x9f\x98\x80", b"\xff", b"\x80", b"\xe2\x82", b" "]
    for trial in range(300):
        raw = b"".join(rng.choice(alphabet) for _ in range(rng.randint(0, 12)))
        cuts = sorted(rng.sample(range(1, len(raw)), min(len(raw) - 1, rng.randint(0, 6)))) if len(raw) > 1 else []
        pieces = [raw[a:b] for a, b in zip([0] + cuts, cuts + [len(raw)])] if raw else []
        io = IncrementalOutput(())
        out = b""
        for pc in pieces:
            d, hit = io.push(pc)
            d.decode("utf-8")                      # valid on its own
            assert not hit
            out += d
        tail = io.finish()
        tail.decode("utf-8")
        assert (out + tail).decode("utf-8") == raw.decode("utf-8", errors="replace"), (raw, pieces)


def _first_stop(full: bytes, stops):
    """Oracle: the start of the stop string that completes first in ``full``
    (the earliest end; on equal ends the longer match), or None."""
    best = None
    for s in stops:
        i = full.find(s)
        while i >= 0:
            end = i + len(s)
            if best is None or end < best[0] or (end == best[0] and i < best[1]):
                best = (end, i)
            i = full.find(s, i + 1)
    return None if best is None else best[1]


def test_incremental_output_stop_strings_split_invariant():
    """Stop strings (overlapping, sharing prefixes, multi-byte) are found at
    the same place however the bytes are cut into token pieces, nothing after
    the stop is released, and without a hit the deltas plus the terminal tail
    are the whole text (reference: service/incremental_output/output_wbtest.mbt,
    'stop text spanning token pieces is withheld before terminal',
    'stop matcher spans UTF-8 bytes')."""
    import random
    rng = random.Random(11)
    alphabet = [b"a", b"b", b"c", b"\xc3\xa9", b"\xe2\x82\xac", b" "]
    stop_sets = [[b"abca"], [b"abcd", b"bc"], [b"aa", b"aab"], ["é€".encode()], [b"ab", "b€".encode(), b"ca c"]]
    for trial in range(400):
        stops = rng.choice(stop_sets)
        full = b"".join(rng.choice(alphabet) for _ in range(rng.randint(0, 16)))
        cuts = sorted(rng.sample(range(1, len(full)), min(len(full) - 1, rng.randint(0, 8)))) if len(full) > 1 else []
        pieces = [full[a:b] for a, b in zip([0] + cuts, cuts + [len(full)])] if full else []
        io = IncrementalOutput(stops)
        out, hit = b"", False
        for pc in pieces:
            d, hit = io.push(pc)
            out += d
            if hit:
                break
        cut = _first_stop(full, stops)
        if cut is None:
            assert not hit
            assert out + io.finish() == full, (stops, pieces)
        else:
            assert hit and out == full[:cut], (stops, pieces, out)
            assert io.finish() == b"" and io.push(b"more") == (b"", True)
