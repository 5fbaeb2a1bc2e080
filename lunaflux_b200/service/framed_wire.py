"""The public framed TCP wire: request v1 and event v2, byte-compatible.

Reference: service/framed_wire/request_codec.mbt:2-174, event_codec.mbt:2-142,
endian.mbt:39-47, types.mbt (header sizes, 16 MiB frame cap).  The layouts are
the reference's because they are the protocol; the code is this framework's.

Common rules: little-endian fixed header; magic, version and kind at 0/4/8;
exact total length at 12; FNV-1a (32-bit) checksum at 16 over every byte
except [16, 20); reserved bytes and unused scalars must be zero.

Request v1 (header 256 bytes):
  20 flags (text=1 sample=2 top_k=4 top_p=8 streaming=16 trace=32)
  24 protocol wire code (1)    28 input count (bytes or tokens)
  32 stop-token count  36 stop-string count  40 stop-string bytes
  44 cache-scope bytes 48 trace bytes  52 max_new_tokens  56 context ceiling
  60 mode (0 greedy, 1 sample)  64 top_k  72 f64 temperature  80 f64 top_p
  88 u64 seed  96 u64 deadline ms  104 u64 request id
  112 / 176 model content / plan digest (64 lowercase hex ASCII each)
  240 cache permission (0 disabled, 1 read-only, 2 read-write)
  244 payload bytes  248 header bytes (256)
  payload: input (UTF-8 or i32 tokens), stop tokens (i32), stop strings
  (u32 length + bytes each), cache scope, trace.
Event v2 (header 208 bytes):
  8 kind (1 Accepted 2 Token 3 Usage 4 Completed 5 Failed)
  20 delta-present flag  24 token id / finish reason (0 stop 1 limit 2
  cancelled) / retryable  28 position  32..44 usage (input, cached input,
  output, total)  48 / 52 Accepted max_new / context ceiling  56 payload bytes
  64 / 128 Accepted content / plan digest  196 header bytes (208)
  payload: token delta, final delta, or the public failure code string.
"""
from __future__ import annotations

import dataclasses
import struct
from typing import List, Optional, Tuple, Union

from ..contracts.inference import (CachePermission, CacheScope, CompletedEvent, ContractError, FailedEvent,
                                   FinishReason, GenerateRequest, InferenceLimits, PublicErrorCode, SamplingMode,
                                   SamplingParameters, StopConditions, TokenEvent, Usage, validate_event)

REQUEST_MAGIC = 0x5152464C
EVENT_MAGIC = 0x5645464C
REQUEST_VERSION = 1
EVENT_VERSION = 2
REQUEST_HEADER = 256
EVENT_HEADER = 208
MAX_FRAME = 16 * 1024 * 1024

F_TEXT, F_SAMPLE, F_TOPK, F_TOPP, F_STREAM, F_TRACE = 1, 2, 4, 8, 16, 32
K_ACCEPTED, K_TOKEN, K_USAGE, K_COMPLETED, K_FAILED = 1, 2, 3, 4, 5
_FINISH_CODE = {FinishReason.STOP_SEQUENCE: 0, FinishReason.TOKEN_LIMIT: 1, FinishReason.CANCELLED: 2}
_FINISH_FROM = {v: k for k, v in _FINISH_CODE.items()}


class FramedWireError(ValueError):
    """Carries only the frame kind and the rule violated, never payload bytes."""

    def __init__(self, frame: str, rule: str):
        super().__init__(f"{frame}:{rule}")
        self.frame = frame
        self.rule = rule


def fnv1a(buf: bytes) -> int:
    h = 2166136261
    for i, b in enumerate(buf):
        if 16 <= i < 20:
            continue
        h = ((h ^ b) * 16777619) & 0xFFFFFFFF
    return h


def _u32(b, o):
    return struct.unpack_from("<I", b, o)[0]


def _i32(b, o):
    return struct.unpack_from("<i", b, o)[0]


def _u64(b, o):
    return struct.unpack_from("<Q", b, o)[0]


def _f64(b, o):
    return struct.unpack_from("<d", b, o)[0]


def _hexdigest_ok(s: bytes) -> bool:
    return len(s) == 64 and all(c in b"0123456789abcdef" for c in s)


# ---------------------------------------------------------------------------
# Request v1
# ---------------------------------------------------------------------------
def encode_request(req: GenerateRequest) -> bytes:
    text = req.input_tokens is None
    inp = req.input_text if text else b"".join(struct.pack("<i", t) for t in req.input_tokens)
    stop_ids = b"".join(struct.pack("<i", t) for t in req.stop.token_ids)
    stop_str = b"".join(struct.pack("<I", len(s)) + s for s in req.stop.strings)
    scope = req.cache.scope
    trace = req.trace or b""
    payload = inp + stop_ids + stop_str + scope + trace
    total = REQUEST_HEADER + len(payload)
    if total > MAX_FRAME:
        raise FramedWireError("request", "too_large")
    h = bytearray(REQUEST_HEADER)
    sp = req.sampling
    flags = (F_TEXT if text else 0) | (F_SAMPLE if sp.mode is SamplingMode.SAMPLE else 0) | \
        (F_TOPK if sp.top_k is not None else 0) | (F_TOPP if sp.top_p is not None else 0) | \
        (F_STREAM if req.streaming else 0) | (F_TRACE if req.trace is not None else 0)
    struct.pack_into("<IIII", h, 0, REQUEST_MAGIC, REQUEST_VERSION, 1, total)
    struct.pack_into("<I", h, 20, flags)
    struct.pack_into("<iiiiiiiiiiii", h, 24, 1, len(req.input_text) if text else len(req.input_tokens),
                     len(req.stop.token_ids), len(req.stop.strings), sum(len(s) for s in req.stop.strings),
                     len(scope), len(trace), req.max_new_tokens, req.context_ceiling or 0,
                     1 if sp.mode is SamplingMode.SAMPLE else 0, sp.top_k or 0, 0)
    struct.pack_into("<ddQQQ", h, 72, sp.temperature, sp.top_p or 0.0, sp.seed, req.deadline_millis or 0,
                     req.request_id)
    for off, dg in ((112, req.model_content_digest), (176, req.model_plan_digest)):
        d = (dg or "0" * 64).encode()
        if not _hexdigest_ok(d):
            raise FramedWireError("request", "digest")
        h[off:off + 64] = d
    struct.pack_into("<iii", h, 240, req.cache.permission.value, len(payload), REQUEST_HEADER)
    frame = bytearray(bytes(h) + payload)
    struct.pack_into("<I", frame, 16, fnv1a(frame))
    return bytes(frame)


def decode_request(frame: bytes, limits: InferenceLimits) -> GenerateRequest:
    def bad(rule):
        raise FramedWireError("request", rule)

    n = len(frame)
    if n < REQUEST_HEADER:
        bad("length")
    if n > MAX_FRAME:
        bad("too_large")
    magic, ver, kind, total = struct.unpack_from("<IIII", frame, 0)
    if magic != REQUEST_MAGIC or kind != 1:
        bad("magic")
    if ver != REQUEST_VERSION:
        bad("version")
    if total != n:
        bad("length")
    if _u32(frame, 16) != fnv1a(frame):
        bad("checksum")
    flags = _u32(frame, 20)
    if flags & ~63:
        bad("flags")
    (proto, n_in, n_stop_ids, n_stop_str, stop_bytes, scope_len, trace_len, max_new, ctx, mode, top_k,
     reserved) = struct.unpack_from("<iiiiiiiiiiii", frame, 24)
    temperature, top_p = _f64(frame, 72), _f64(frame, 80)
    seed, deadline, rid = _u64(frame, 88), _u64(frame, 96), _u64(frame, 104)
    perm, payload_len, hdr = struct.unpack_from("<iii", frame, 240)
    if proto != 1:
        bad("protocol")
    if reserved != 0 or any(frame[252:256]):
        bad("reserved")
    if hdr != REQUEST_HEADER or payload_len != n - REQUEST_HEADER:
        bad("length")
    if min(n_in, n_stop_ids, n_stop_str, stop_bytes, scope_len, trace_len) < 0:
        bad("count")
    if n_in > max(limits.max_text_bytes, limits.max_input_tokens) or n_stop_ids > limits.max_stop_token_ids or \
            n_stop_str > limits.max_stop_strings:
        bad("count")
    sample = bool(flags & F_SAMPLE)
    if (mode == 1) != sample or mode not in (0, 1):
        bad("mode")
    if not (flags & F_TOPK) and top_k != 0:
        bad("unused_scalar")
    if not (flags & F_TOPP) and struct.unpack_from("<Q", frame, 80)[0] != 0:
        bad("unused_scalar")
    if not (flags & F_TRACE) and trace_len != 0:
        bad("unused_scalar")
    try:
        perm_e = CachePermission(perm)
    except ValueError:
        bad("cache_permission")
    digests = []
    for off in (112, 176):
        d = bytes(frame[off:off + 64])
        if not _hexdigest_ok(d):
            bad("digest")
        digests.append("" if d == b"0" * 64 else d.decode())
    cur = REQUEST_HEADER
    text = bool(flags & F_TEXT)
    in_bytes = n_in if text else 4 * n_in
    if cur + in_bytes > n:
        bad("payload")
    if text:
        input_text, input_tokens = bytes(frame[cur:cur + n_in]), None
    else:
        input_text, input_tokens = None, tuple(struct.unpack_from(f"<{n_in}i", frame, cur))
    cur += in_bytes
    if cur + 4 * n_stop_ids > n:
        bad("payload")
    stop_ids = tuple(struct.unpack_from(f"<{n_stop_ids}i", frame, cur))
    cur += 4 * n_stop_ids
    strings = []
    total_str = 0
    for _ in range(n_stop_str):
        if cur + 4 > n:
            bad("payload")
        ln = _u32(frame, cur)
        cur += 4
        if ln > limits.max_stop_string_bytes or cur + ln > n:
            bad("payload")
        strings.append(bytes(frame[cur:cur + ln]))
        cur += ln
        total_str += ln
    if total_str != stop_bytes:
        bad("payload")
    if cur + scope_len + trace_len != n:
        bad("payload")
    scope = bytes(frame[cur:cur + scope_len])
    cur += scope_len
    trace = bytes(frame[cur:cur + trace_len]) if flags & F_TRACE else None
    sp = SamplingParameters(SamplingMode.SAMPLE if sample else SamplingMode.GREEDY, temperature,
                            top_k if flags & F_TOPK else None, top_p if flags & F_TOPP else None, seed)
    req = GenerateRequest(request_id=rid, input_tokens=input_tokens, input_text=input_text, max_new_tokens=max_new,
                          context_ceiling=ctx or None, sampling=sp, stop=StopConditions(stop_ids, tuple(strings)),
                          streaming=bool(flags & F_STREAM), deadline_millis=deadline or None,
                          cache=CacheScope(scope, perm_e), trace=trace, model_content_digest=digests[0],
                          model_plan_digest=digests[1])
    try:
        return req.validate(limits)
    except ContractError as e:
        raise FramedWireError("request", f"contract:{e.field.name}") from None


# ---------------------------------------------------------------------------
# Event v2
# ---------------------------------------------------------------------------
@dataclasses.dataclass(frozen=True)
class AcceptedWire:
    request_id: int
    max_new_tokens: int
    context_ceiling: int
    content_digest: str = ""
    plan_digest: str = ""


Event = Union[AcceptedWire, TokenEvent, Usage, CompletedEvent, FailedEvent]


def _usage_into(h, u: Usage):
    struct.pack_into("<iiii", h, 32, u.input_tokens, u.cached_input_tokens, u.output_tokens, u.total_tokens)


def encode_event(ev: Event) -> bytes:
    if not isinstance(ev, AcceptedWire):
        try:
            validate_event(ev)
        except ContractError as e:
            raise FramedWireError("event", f"contract:{e.field.name}") from None
    h = bytearray(EVENT_HEADER)
    payload = b""
    if isinstance(ev, AcceptedWire):
        kind = K_ACCEPTED
        struct.pack_into("<ii", h, 48, ev.max_new_tokens, ev.context_ceiling)
        for off, dg in ((64, ev.content_digest), (128, ev.plan_digest)):
            d = (dg or "0" * 64).encode()
            if not _hexdigest_ok(d):
                raise FramedWireError("event", "digest")
            h[off:off + 64] = d
    elif isinstance(ev, TokenEvent):
        kind = K_TOKEN
        struct.pack_into("<ii", h, 24, ev.token_id, ev.position)
        if ev.delta:
            payload = ev.delta
            struct.pack_into("<I", h, 20, 1)
    elif isinstance(ev, Usage):
        kind = K_USAGE
        _usage_into(h, ev)
    elif isinstance(ev, CompletedEvent):
        kind = K_COMPLETED
        struct.pack_into("<i", h, 24, _FINISH_CODE[ev.reason])
        _usage_into(h, ev.usage)
        if ev.final_delta:
            payload = ev.final_delta
            struct.pack_into("<I", h, 20, 1)
    elif isinstance(ev, FailedEvent):
        kind = K_FAILED
        struct.pack_into("<i", h, 24, 1 if ev.retryable else 0)
        payload = ev.code.value.encode()
    else:
        raise FramedWireError("event", "kind")
    total = EVENT_HEADER + len(payload)
    if total > MAX_FRAME:
        raise FramedWireError("event", "too_large")
    struct.pack_into("<IIiI", h, 0, EVENT_MAGIC, EVENT_VERSION, kind, total)
    struct.pack_into("<i", h, 56, len(payload))
    struct.pack_into("<i", h, 196, EVENT_HEADER)
    frame = bytearray(bytes(h) + payload)
    struct.pack_into("<I", frame, 16, fnv1a(frame))
    return bytes(frame)


def decode_event(frame: bytes, request_id: int = 0) -> Event:
    def bad(rule):
        raise FramedWireError("event", rule)

    n = len(frame)
    if n < EVENT_HEADER or n > MAX_FRAME:
        bad("length")
    magic, ver, kind, total = struct.unpack_from("<IIiI", frame, 0)
    if magic != EVENT_MAGIC:
        bad("magic")
    if ver != EVENT_VERSION:
        bad("version")
    if total != n or _i32(frame, 196) != EVENT_HEADER or _i32(frame, 56) != n - EVENT_HEADER:
        bad("length")
    if _u32(frame, 16) != fnv1a(frame):
        bad("checksum")
    payload = bytes(frame[EVENT_HEADER:])
    flag = _u32(frame, 20)
    if flag not in (0, 1):
        bad("flags")

    def zero(a, b):
        if any(frame[a:b]):
            bad("reserved")

    def usage():
        i, c, o, t = struct.unpack_from("<iiii", frame, 32)
        if min(i, c, o) < 0 or c > i or t != i + o:
            bad("usage")
        return Usage(i, c, o)

    if kind == K_ACCEPTED:
        zero(20, 48)
        zero(192, 196)
        zero(200, 208)
        digs = []
        for off in (64, 128):
            d = bytes(frame[off:off + 64])
            if not _hexdigest_ok(d):
                bad("digest")
            digs.append("" if d == b"0" * 64 else d.decode())
        if payload:
            bad("payload")
        return AcceptedWire(request_id, _i32(frame, 48), _i32(frame, 52), digs[0], digs[1])
    if kind == K_TOKEN:
        zero(32, 56)
        zero(60, 196)
        if bool(flag) != bool(payload):
            bad("payload")
        return TokenEvent(request_id, _i32(frame, 28), _i32(frame, 24), payload)
    if kind == K_USAGE:
        zero(20, 32)
        zero(48, 56)
        zero(60, 196)
        if payload:
            bad("payload")
        return usage()
    if kind == K_COMPLETED:
        zero(28, 32)
        zero(48, 56)
        zero(60, 196)
        if bool(flag) != bool(payload):
            bad("payload")
        code = _i32(frame, 24)
        if code not in _FINISH_FROM:
            bad("finish_reason")
        return CompletedEvent(request_id, _FINISH_FROM[code], usage(), payload)
    if kind == K_FAILED:
        zero(28, 56)
        zero(60, 196)
        r = _i32(frame, 24)
        if r not in (0, 1) or flag:
            bad("scalar")
        try:
            code = PublicErrorCode(payload.decode("ascii"))
        except (ValueError, UnicodeDecodeError):
            bad("public_code")
        return FailedEvent(request_id, code, bool(r))
    bad("kind")


class FrameReader:
    """Incremental splitter: feed bytes, take complete frames (length at 12)."""

    def __init__(self, magic: int, max_frame: int = MAX_FRAME, header: int = REQUEST_HEADER):
        self.magic = magic
        self.max_frame = max_frame
        self.header = header
        self.buf = bytearray()
        self.poisoned = False
        self._first = 0.0        # receipt time of the first buffered byte

    @property
    def first_byte_time(self) -> float:
        """Receipt time (as passed to ``feed_timed``) of the buffered partial frame."""
        return self._first

    def feed(self, data: bytes) -> List[bytes]:
        if self.poisoned:
            raise FramedWireError("stream", "poisoned")
        self.buf += data
        out = []
        while len(self.buf) >= 16:
            magic, _, _, total = struct.unpack_from("<IIII", self.buf, 0)
            if magic != self.magic or total < self.header or total > self.max_frame:
                self.poisoned = True
                raise FramedWireError("stream", "prefix")
            if len(self.buf) < total:
                break
            out.append(bytes(self.buf[:total]))
            del self.buf[:total]
        return out

    def feed_timed(self, data: bytes, now: float) -> List[Tuple[bytes, float]]:
        """As ``feed``, with each frame's receipt time: the time passed with
        the chunk that carried the frame's first byte.  The first frame a
        chunk completes may have started in an earlier chunk; every later one
        started in this chunk (the frame before it ended here)."""
        if not self.buf and data:
            self._first = now
        frames = self.feed(data)
        out = []
        for i, f in enumerate(frames):
            out.append((f, self._first if i == 0 else now))
        if frames:
            self._first = now     # the bytes left over (if any) arrived in this chunk
        return out
