"""Wire compatibility with the reference's frozen frames.

The reference pins the SHA-256 of two canonical frames in its own tests:
the request-v1 frame of its codec fixture (service/framed_wire/
codec_wbtest.mbt:75-103: request 42, text "hello moon", sample T 0.75 /
top-k 12 / top-p 0.9 / seed 99, stops [2, 7] + ["END", "stop"], deadline
5000 ms, scope "tenant-a", trace "trace-7", 304 bytes) and the event-v2
Accepted frame of the same fixture identity (codec_wbtest.mbt:271-330,
luna_event_adapter_wbtest.mbt:36-40, 208 bytes).  This codec, written from
the documented layout, must produce those exact bytes and read them back
field for field, whole or split at any byte.
"""
import hashlib
import struct

import pytest

from lunaflux_b200.contracts.inference import (CachePermission, CacheScope, CompletedEvent, FailedEvent,
                                               FinishReason, GenerateRequest, InferenceLimits, PublicErrorCode,
                                               SamplingParameters, StopConditions, TokenEvent, Usage)
from lunaflux_b200.service.framed_wire import (EVENT_HEADER, EVENT_MAGIC, REQUEST_MAGIC, AcceptedWire, FrameReader,
                                               FramedWireError, decode_event, decode_request, encode_event,
                                               encode_request, fnv1a)

REQUEST_SHA256 = "09e534bb3c7d1b9200362b23239dc5c11352ae50811313c800bbe6c717efa72f"
ACCEPTED_SHA256 = "341ae02aa5d3160f35595d8e4a091e1ef299679d08f1ce6c565bb35d8b288c71"
CONTENT = "0123456789abcdef" * 4
PLAN = "abcdef0123456789" * 4

LIM = InferenceLimits(max_text_bytes=64, max_input_tokens=16, max_new_tokens=12, max_context_tokens=32,
                      max_token_id=255, max_stop_token_ids=4, max_stop_strings=3, max_stop_string_bytes=16,
                      max_trace_bytes=16, max_cache_scope_bytes=16, max_decoded_delta_bytes=16,
                      max_deadline_millis=10000, max_top_k=256, max_temperature=8.0)


def fixture_request():
    return GenerateRequest(42, input_text=b"hello moon", max_new_tokens=4, context_ceiling=16,
                           sampling=SamplingParameters.sample(0.75, top_k=12, top_p=0.9, seed=99),
                           stop=StopConditions((2, 7), (b"END", b"stop")), streaming=True, deadline_millis=5000,
                           cache=CacheScope(b"tenant-a", CachePermission.READ_WRITE), trace=b"trace-7",
                           model_content_digest=CONTENT, model_plan_digest=PLAN)


def sha(b):
    return hashlib.sha256(b).hexdigest()


def refresh(b: bytearray) -> bytes:
    struct.pack_into("<I", b, 16, 0)
    struct.pack_into("<I", b, 16, fnv1a(bytes(b)))
    return bytes(b)


def test_request_frame_equals_the_reference_golden():
    frame = encode_request(fixture_request())
    assert len(frame) == 304 and sha(frame) == REQUEST_SHA256
    back = decode_request(frame, LIM)
    assert back == fixture_request()
    assert back.input_text.decode() == "hello moon" and back.stop.strings[1] == b"stop"
    assert back.sampling.top_k == 12 and back.sampling.top_p == 0.9 and back.sampling.seed == 99
    assert back.cache.scope == b"tenant-a" and back.trace == b"trace-7"


def test_accepted_frame_equals_the_reference_golden():
    frame = encode_event(AcceptedWire(42, 4, 16, CONTENT, PLAN))
    assert len(frame) == EVENT_HEADER == 208 and sha(frame) == ACCEPTED_SHA256
    assert decode_event(frame, 42) == AcceptedWire(42, 4, 16, CONTENT, PLAN)


def test_golden_request_at_every_split_point():
    frame = encode_request(fixture_request())
    for split in range(len(frame) + 1):
        rd = FrameReader(REQUEST_MAGIC, 4096)
        got = rd.feed(frame[:split]) + rd.feed(frame[split:])
        assert got == [frame], split
        assert not rd.buf


def test_golden_request_bytewise_then_a_pipelined_second_frame():
    frame = encode_request(fixture_request())
    rd = FrameReader(REQUEST_MAGIC, 4096)
    out = []
    for i in range(len(frame)):
        out += rd.feed(frame[i:i + 1])
        assert out == ([] if i < len(frame) - 1 else [frame])
    # a frame followed by the first bytes of the next: the tail stays buffered
    out = rd.feed(frame + frame[:10])
    assert out == [frame] and bytes(rd.buf) == frame[:10]


def test_all_event_variants_roundtrip():
    usage = Usage(3, 1, 2)
    assert usage.total_tokens == 5
    events = [AcceptedWire(42, 4, 16, CONTENT, PLAN), TokenEvent(42, 1, 9, b"ok"), usage,
              CompletedEvent(42, FinishReason.TOKEN_LIMIT, usage, b"tail"),
              FailedEvent(42, PublicErrorCode.WORKER_UNAVAILABLE, True)]
    for ev in events:
        frame = encode_event(ev)
        assert decode_event(frame, 42) == ev
        rd = FrameReader(EVENT_MAGIC, 4096, header=EVENT_HEADER)
        assert rd.feed(frame[:7]) + rd.feed(frame[7:]) == [frame]


@pytest.mark.parametrize("what,offset,fmt,value", [
    ("usage total disagrees", 44, "<i", 99),            # input + output != total
    ("cached above input", 36, "<i", 9),
    ("token flag without payload", 20, "<I", 1),
    ("unknown kind", 8, "<i", 77),
    ("reserved byte set", 100, "<B", 1),
])
def test_event_semantic_mutation_with_refreshed_checksum_is_rejected(what, offset, fmt, value):
    ev = Usage(3, 1, 2) if "usage" in what or "cached" in what else TokenEvent(42, 1, 9, b"")
    b = bytearray(encode_event(ev))
    struct.pack_into(fmt, b, offset, value)
    with pytest.raises(FramedWireError):
        decode_event(refresh(b), 42)


@pytest.mark.parametrize("offset,value", [
    (28, 1 << 30),       # input count
    (32, 1 << 30),       # stop token count
    (36, 1 << 30),       # stop string count
    (40, 1 << 30),       # stop string bytes
    (44, -1),            # cache scope length
    (48, 1 << 30),       # trace length
])
def test_hostile_request_counts_reject_before_allocation(offset, value):
    b = bytearray(encode_request(fixture_request()))
    struct.pack_into("<i", b, offset, value)
    with pytest.raises(FramedWireError):
        decode_request(refresh(b), LIM)


def test_request_trailing_bytes_and_truncation_reject():
    frame = encode_request(fixture_request())
    for bad in (frame + b"\x00", frame[:-1]):
        with pytest.raises(FramedWireError):
            decode_request(bad, LIM)
    # the length word disagrees with the payload it carries
    b = bytearray(frame)
    struct.pack_into("<I", b, 12, len(frame) - 1)
    with pytest.raises(FramedWireError):
        decode_request(refresh(b), LIM)
