"""Rank-control wire frames: exact round trips and typed rejection of every
corruption (the reference's worker_wire corruption tables:
engine/worker_wire/plan_corruption_wbtest.mbt, completion_corruption_wbtest.mbt)."""
import math
import struct

import pytest

from lunaflux_b200.contracts import SamplingMode, SamplingParameters
from lunaflux_b200.engine import worker_wire as ww

MESSAGES = [
    ("ready", 3),
    ("hb", 1, 12345.625),
    ("add", 7, [1, 2, 3, 128000], 16, SamplingParameters(), ()),
    ("add", 2**40, list(range(1000)), 1, SamplingParameters(SamplingMode.SAMPLE, 0.7, 40, 0.9, 99), (5, 6)),
    ("add", 0, [], 0, SamplingParameters(SamplingMode.SAMPLE, 1.0, None, None, 1), ()),
    ("cancel", 11),
    ("step", 1234.5),
    ("close",),
    ("outs", 0, [(1, 42, False), (2, 7, True)], [(2, "TOKEN_LIMIT", None), (9, None, "WORKER_UNAVAILABLE")], True),
    ("outs", 5, [], [], False),
    ("error", 1, "Traceback: boom ü"),
]


@pytest.mark.parametrize("msg", MESSAGES, ids=[m[0] + str(i) for i, m in enumerate(MESSAGES)])
def test_round_trip(msg):
    frame = ww.encode(msg, generation=4)
    back, gen = ww.decode_with_generation(frame)
    assert gen == 4
    assert back == msg


def _issue(frame):
    with pytest.raises(ww.WireError) as e:
        ww.decode(frame)
    return e.value.issue


@pytest.mark.parametrize("msg", MESSAGES, ids=[m[0] + str(i) for i, m in enumerate(MESSAGES)])
def test_every_truncation_is_rejected(msg):
    frame = ww.encode(msg)
    for n in range(len(frame)):
        assert _issue(frame[:n]) in (ww.WireIssue.TRUNCATED, ww.WireIssue.LENGTH_MISMATCH)


@pytest.mark.parametrize("msg", MESSAGES, ids=[m[0] + str(i) for i, m in enumerate(MESSAGES)])
def test_trailing_bytes_are_rejected(msg):
    frame = bytearray(ww.encode(msg)) + b"\0"
    struct.pack_into("<I", frame, 8, len(frame) - ww.HEADER_BYTES)   # a consistent length field
    assert _issue(bytes(frame)) is ww.WireIssue.TRAILING_BYTES


def test_header_corruptions():
    frame = bytearray(ww.encode(("close",)))
    bad = bytearray(frame)
    bad[0] ^= 1
    assert _issue(bytes(bad)) is ww.WireIssue.BAD_MAGIC
    bad = bytearray(frame)
    struct.pack_into("<H", bad, 4, 2)
    assert _issue(bytes(bad)) is ww.WireIssue.BAD_VERSION
    for k in (0, 9, 0xFFFF):
        bad = bytearray(frame)
        struct.pack_into("<H", bad, 6, k)
        assert _issue(bytes(bad)) is ww.WireIssue.UNKNOWN_KIND
    bad = bytearray(frame)
    struct.pack_into("<I", bad, 8, 1)
    assert _issue(bytes(bad)) is ww.WireIssue.LENGTH_MISMATCH


def test_field_corruptions():
    add = bytearray(ww.encode(("add", 1, [1, 2], 4, SamplingParameters(), ())))
    off = ww.HEADER_BYTES + 8 + 4          # sampling mode byte
    bad = bytearray(add)
    bad[off] = 7
    assert _issue(bytes(bad)) is ww.WireIssue.BAD_VALUE
    bad = bytearray(add)
    struct.pack_into("<d", bad, off + 1, math.inf)    # temperature
    assert _issue(bytes(bad)) is ww.WireIssue.BAD_VALUE
    bad = bytearray(add)
    struct.pack_into("<d", bad, off + 13, 1.5)        # top_p
    assert _issue(bytes(bad)) is ww.WireIssue.BAD_VALUE
    bad = bytearray(add)
    struct.pack_into("<I", bad, off + 29, ww.MAX_PROMPT_TOKENS + 1)   # prompt count beyond the limit
    assert _issue(bytes(bad)) is ww.WireIssue.LIMIT
    outs = bytearray(ww.encode(("outs", 0, [(1, 2, True)], [(1, "CANCELLED", None)], False)))
    bad = bytearray(outs)
    bad[ww.HEADER_BYTES + 4] = 2                      # has_work flag
    assert _issue(bytes(bad)) is ww.WireIssue.BAD_VALUE
    bad = bytearray(outs)
    bad[ww.HEADER_BYTES + 5 + 4 + 12] = 3             # finished flag
    assert _issue(bytes(bad)) is ww.WireIssue.BAD_VALUE
    bad = bytearray(outs)
    bad[-2] = 99                                      # finish reason code
    assert _issue(bytes(bad)) is ww.WireIssue.BAD_VALUE


def test_encode_rejects_invalid_messages():
    for msg in [("bogus",), ("cancel", -1), ("add", 1, [0] * (ww.MAX_STOP_IDS + 1), 1, None, ()),
                ("add", 1, [1], 1, None, tuple(range(ww.MAX_STOP_IDS + 1)))]:
        if msg[0] == "add" and len(msg[2]) <= ww.MAX_PROMPT_TOKENS and len(msg[5]) <= ww.MAX_STOP_IDS:
            continue
        with pytest.raises(ww.WireError):
            ww.encode(msg)


def test_channel_rejects_a_stale_generation():
    import socket
    from lunaflux_b200.engine.channel import MessageChannel
    a, b = socket.socketpair()
    ca, cb = MessageChannel(a), MessageChannel(b)
    ca.generation, cb.generation = 2, 2
    ca.send(("step", 1.0))
    assert cb.recv(5.0) == ("step", 1.0)
    ca.generation = 1
    ca.send(("step", 2.0))
    with pytest.raises(EOFError):
        cb.recv(5.0)
    ca.close()
    cb.close()


GOLDEN = [
    (("cancel", 11), "4c4c46570100040008000000030000000b00000000000000"),
    (("step", 1234.5), "4c4c465701000500080000000300000000000000004a9340"),
    (("close",), "4c4c4657010006000000000003000000"),
    (("add", 7, [1, 2, 3], 16, SamplingParameters(SamplingMode.SAMPLE, 0.5, 40, 0.75, 99), (5,)),
     "4c4c465701000300410000000300000007000000000000001000000001000000000000e03f28000000000000000000e83f63"
     "00000000000000030000000100000002000000030000000100000005000000"),
    (("outs", 2, [(1, 42, False)], [(9, None, "WORKER_UNAVAILABLE")], True),
     "4c4c465701000700240000000300000002000000010100000001000000000000002a000000000100000009000000000000"
     "000004"),
]


@pytest.mark.parametrize("msg,hexbytes", GOLDEN, ids=[g[0][0] for g in GOLDEN])
def test_golden_bytes(msg, hexbytes):
    """The encoding is byte-for-byte deterministic and pinned: a change of
    layout, of a kind tag or of a reason / error tag shows up here
    (reference: 'canonical encoding is byte-for-byte deterministic', 'wire
    tags are pinned independently in both directions')."""
    assert ww.encode(msg, generation=3).hex() == hexbytes
    assert ww.decode_with_generation(bytes.fromhex(hexbytes)) == (msg, 3)


def test_tags_are_pinned_in_both_directions():
    from lunaflux_b200.contracts import FinishReason, PublicErrorCode
    kinds = {"READY": 1, "HEARTBEAT": 2, "ADD": 3, "CANCEL": 4, "STEP": 5, "CLOSE": 6, "OUTPUTS": 7, "ERROR": 8}
    assert {k.name: int(k) for k in ww.Kind} == kinds
    assert [None if r is None else r.name for r in ww._REASONS] == [None, "STOP_SEQUENCE", "TOKEN_LIMIT", "CANCELLED"]
    assert [None if e is None else e.name for e in ww._ERRORS] == [
        None, "INVALID_REQUEST", "OVERLOADED", "DEADLINE_EXCEEDED", "WORKER_UNAVAILABLE", "INTERNAL",
        "CONTEXT_OVERFLOW", "CANCELLED"]
    assert set(ww._REASONS[1:]) == set(FinishReason) and set(ww._ERRORS[1:]) == set(PublicErrorCode)
