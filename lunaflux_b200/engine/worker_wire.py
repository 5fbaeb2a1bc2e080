"""Binary frames of the rank-control protocol (supervisor <-> rank workers).

Reference: engine/worker_wire (fixed little-endian plan / completion /
startup frames with magic numbers, versions and structural validation; every
corruption is rejected with a typed error: plan_corruption_wbtest.mbt,
completion_corruption_wbtest.mbt).  The reference ships whole step plans to a
stateless executor; here every rank runs the same deterministic scheduler, so
the frames carry the *commands* that change the schedulers (admit, cancel,
step, close), the ranks' completions and their start-up / liveness reports.
The layouts below are this project's own.

Every frame is

    offset  size  field
    0       4     magic   0x57464C4C ("LLFW" little-endian)
    4       2     version (1)
    6       2     kind    (Kind)
    8       4     payload length in bytes
    12      4     generation of the rank group the frame belongs to
    16      ...   payload (kind-specific, little-endian, no padding)

followed by nothing: trailing bytes are an error.  The framed channel around
it (``engine/channel.py``) adds the length prefix and an FNV-1a checksum, so a
frame that reaches ``decode`` was transmitted intact; ``decode`` still
validates every field, so a buggy or hostile peer cannot make it allocate
without bound or produce an out-of-range value.

Messages are the supervisor's tuples (``("add", rid, prompt, max_new,
sampling, stop_ids)`` and so on): ``encode(msg)`` / ``decode(frame)`` are exact
inverses for every valid message.
"""
from __future__ import annotations

import enum
import math
import struct
from typing import Optional, Tuple

from ..contracts import FinishReason, PublicErrorCode, SamplingMode, SamplingParameters

MAGIC = 0x57464C4C
VERSION = 1
HEADER = struct.Struct("<IHHII")
HEADER_BYTES = HEADER.size          # 16

MAX_PROMPT_TOKENS = 1 << 20
MAX_STOP_IDS = 256
MAX_OUTPUTS = 1 << 16
MAX_ERROR_BYTES = 8192
MAX_FRAME_BYTES = HEADER_BYTES + 16 * MAX_OUTPUTS * 2 + 4 * MAX_PROMPT_TOKENS + 64


class Kind(enum.IntEnum):
    READY = 1        # rank -> supervisor: engine built
    HEARTBEAT = 2    # rank -> supervisor: liveness
    ADD = 3          # supervisor -> rank: admit a request
    CANCEL = 4       # supervisor -> rank: cancel a request
    STEP = 5         # supervisor -> rank: run one engine iteration at the supervisor's clock
    CLOSE = 6        # supervisor -> rank: leave
    OUTPUTS = 7      # rank -> supervisor: one iteration's tokens and terminals
    ERROR = 8        # rank -> supervisor: the rank failed (traceback text)


_NAMES = {Kind.READY: "ready", Kind.HEARTBEAT: "hb", Kind.ADD: "add", Kind.CANCEL: "cancel", Kind.STEP: "step",
          Kind.CLOSE: "close", Kind.OUTPUTS: "outs", Kind.ERROR: "error"}
_KINDS = {v: k for k, v in _NAMES.items()}

# finish reasons and error codes as one byte each (0 = none)
_REASONS = [None] + list(FinishReason)
_ERRORS = [None] + list(PublicErrorCode)


class WireIssue(enum.Enum):
    TRUNCATED = "truncated"
    BAD_MAGIC = "bad_magic"
    BAD_VERSION = "bad_version"
    UNKNOWN_KIND = "unknown_kind"
    LENGTH_MISMATCH = "length_mismatch"
    TRAILING_BYTES = "trailing_bytes"
    LIMIT = "limit"
    BAD_VALUE = "bad_value"


class WireError(ValueError):
    def __init__(self, issue: WireIssue, detail: str = ""):
        super().__init__(f"worker wire: {issue.value}" + (f" ({detail})" if detail else ""))
        self.issue = issue


# ------------------------------------------------------------------ writer
class _W:
    def __init__(self):
        self.parts = []

    def u8(self, v):
        self.parts.append(struct.pack("<B", v))

    def u32(self, v):
        self.parts.append(struct.pack("<I", v))

    def i32(self, v):
        self.parts.append(struct.pack("<i", v))

    def u64(self, v):
        self.parts.append(struct.pack("<Q", v))

    def f32(self, v):
        self.parts.append(struct.pack("<f", v))

    def f64(self, v):
        self.parts.append(struct.pack("<d", v))

    def i32s(self, xs, limit):
        xs = list(xs)
        if len(xs) > limit:
            raise WireError(WireIssue.LIMIT, f"{len(xs)} > {limit}")
        self.u32(len(xs))
        self.parts.append(struct.pack(f"<{len(xs)}i", *xs))

    def bytes(self):
        return b"".join(self.parts)


# ------------------------------------------------------------------ reader
class _R:
    def __init__(self, buf: memoryview):
        self.buf = buf
        self.off = 0

    def _take(self, n):
        if self.off + n > len(self.buf):
            raise WireError(WireIssue.TRUNCATED, f"need {n} bytes at {self.off}")
        v = self.buf[self.off:self.off + n]
        self.off += n
        return v

    def u8(self):
        return self._take(1)[0]

    def u32(self):
        return struct.unpack("<I", self._take(4))[0]

    def i32(self):
        return struct.unpack("<i", self._take(4))[0]

    def u64(self):
        return struct.unpack("<Q", self._take(8))[0]

    def f32(self):
        return struct.unpack("<f", self._take(4))[0]

    def f64(self):
        return struct.unpack("<d", self._take(8))[0]

    def i32s(self, limit):
        n = self.u32()
        if n > limit:
            raise WireError(WireIssue.LIMIT, f"{n} > {limit}")
        return list(struct.unpack(f"<{n}i", self._take(4 * n)))

    def end(self):
        if self.off != len(self.buf):
            raise WireError(WireIssue.TRAILING_BYTES, f"{len(self.buf) - self.off} bytes")


def _sampling_out(w: _W, s: Optional[SamplingParameters]):
    s = s or SamplingParameters()
    w.u8(s.mode.value)
    w.f64(s.temperature)
    w.i32(-1 if s.top_k is None else s.top_k)
    w.f64(math.nan if s.top_p is None else s.top_p)
    w.u64(s.seed)


def _sampling_in(r: _R) -> SamplingParameters:
    mode = r.u8()
    if mode not in (0, 1):
        raise WireError(WireIssue.BAD_VALUE, f"sampling mode {mode}")
    temperature = r.f64()
    top_k = r.i32()
    top_p = r.f64()
    seed = r.u64()
    if not math.isfinite(temperature) or (top_k < -1) or (not math.isnan(top_p) and not 0.0 < top_p <= 1.0):
        raise WireError(WireIssue.BAD_VALUE, "sampling parameters")
    return SamplingParameters(SamplingMode(mode), temperature, None if top_k == -1 else top_k,
                              None if math.isnan(top_p) else top_p, seed)


def _nonneg(v, what):
    if not isinstance(v, int) or v < 0:
        raise WireError(WireIssue.BAD_VALUE, f"{what} {v!r}")
    return v


def encode(msg: Tuple, generation: int = 0) -> bytes:
    """The frame of a supervisor / rank message tuple."""
    if not msg or msg[0] not in _KINDS:
        raise WireError(WireIssue.UNKNOWN_KIND, repr(msg[:1]))
    kind = _KINDS[msg[0]]
    w = _W()
    if kind is Kind.READY:
        w.u32(_nonneg(msg[1], "rank"))
    elif kind is Kind.HEARTBEAT:
        w.u32(_nonneg(msg[1], "rank"))
        w.f64(float(msg[2]))
    elif kind is Kind.ADD:
        _, rid, prompt, max_new, sampling, stop_ids = msg
        w.u64(_nonneg(rid, "rid"))
        w.u32(_nonneg(max_new, "max_new"))
        _sampling_out(w, sampling)
        w.i32s(prompt, MAX_PROMPT_TOKENS)
        w.i32s(stop_ids or (), MAX_STOP_IDS)
    elif kind is Kind.CANCEL:
        w.u64(_nonneg(msg[1], "rid"))
    elif kind is Kind.STEP:
        w.f64(float(msg[1]))
    elif kind is Kind.CLOSE:
        pass
    elif kind is Kind.OUTPUTS:
        _, rank, outs, done, has_work = msg
        w.u32(_nonneg(rank, "rank"))
        w.u8(1 if has_work else 0)
        if len(outs) > MAX_OUTPUTS or len(done) > MAX_OUTPUTS:
            raise WireError(WireIssue.LIMIT, "outputs")
        w.u32(len(outs))
        for rid, token, finished in outs:
            w.u64(_nonneg(rid, "rid"))
            w.i32(token)
            w.u8(1 if finished else 0)
        w.u32(len(done))
        for rid, reason, error in done:
            w.u64(_nonneg(rid, "rid"))
            w.u8(0 if reason is None else _REASONS.index(FinishReason[reason]))
            w.u8(0 if error is None else _ERRORS.index(PublicErrorCode[error]))
    elif kind is Kind.ERROR:
        text = str(msg[2]).encode("utf-8")[:MAX_ERROR_BYTES]
        w.u32(_nonneg(msg[1], "rank"))
        w.u32(len(text))
        w.parts.append(text)
    payload = w.bytes()
    return HEADER.pack(MAGIC, VERSION, int(kind), len(payload), generation & 0xFFFFFFFF) + payload


def decode_with_generation(frame) -> Tuple[Tuple, int]:
    """(message tuple, generation) of a frame; WireError if it is malformed."""
    buf = memoryview(bytes(frame))
    if len(buf) < HEADER_BYTES:
        raise WireError(WireIssue.TRUNCATED, "header")
    if len(buf) > MAX_FRAME_BYTES:
        raise WireError(WireIssue.LIMIT, "frame bytes")
    magic, version, kind_v, length, generation = HEADER.unpack_from(buf, 0)
    if magic != MAGIC:
        raise WireError(WireIssue.BAD_MAGIC, hex(magic))
    if version != VERSION:
        raise WireError(WireIssue.BAD_VERSION, str(version))
    try:
        kind = Kind(kind_v)
    except ValueError:
        raise WireError(WireIssue.UNKNOWN_KIND, str(kind_v)) from None
    if length != len(buf) - HEADER_BYTES:
        raise WireError(WireIssue.LENGTH_MISMATCH, f"{length} != {len(buf) - HEADER_BYTES}")
    r = _R(buf[HEADER_BYTES:])
    name = _NAMES[kind]
    if kind is Kind.READY:
        msg = (name, r.u32())
    elif kind is Kind.HEARTBEAT:
        rank = r.u32()
        msg = (name, rank, r.f64())
    elif kind is Kind.ADD:
        rid = r.u64()
        max_new = r.u32()
        sampling = _sampling_in(r)
        prompt = r.i32s(MAX_PROMPT_TOKENS)
        stop_ids = tuple(r.i32s(MAX_STOP_IDS))
        msg = (name, rid, prompt, max_new, sampling, stop_ids)
    elif kind is Kind.CANCEL:
        msg = (name, r.u64())
    elif kind is Kind.STEP:
        msg = (name, r.f64())
    elif kind is Kind.CLOSE:
        msg = (name,)
    elif kind is Kind.OUTPUTS:
        rank = r.u32()
        hw = r.u8()
        if hw > 1:
            raise WireError(WireIssue.BAD_VALUE, "has_work")
        n = r.u32()
        if n > MAX_OUTPUTS:
            raise WireError(WireIssue.LIMIT, "outputs")
        outs = []
        for _ in range(n):
            rid, tok, fin = r.u64(), r.i32(), r.u8()
            if fin > 1:
                raise WireError(WireIssue.BAD_VALUE, "finished flag")
            outs.append((rid, tok, bool(fin)))
        n = r.u32()
        if n > MAX_OUTPUTS:
            raise WireError(WireIssue.LIMIT, "terminals")
        done = []
        for _ in range(n):
            rid, rc, ec = r.u64(), r.u8(), r.u8()
            if rc >= len(_REASONS) or ec >= len(_ERRORS):
                raise WireError(WireIssue.BAD_VALUE, "terminal code")
            done.append((rid, None if rc == 0 else _REASONS[rc].name, None if ec == 0 else _ERRORS[ec].name))
        msg = (name, rank, outs, done, bool(hw))
    else:  # ERROR
        rank = r.u32()
        n = r.u32()
        if n > MAX_ERROR_BYTES:
            raise WireError(WireIssue.LIMIT, "error text")
        text = bytes(r._take(n)).decode("utf-8", errors="replace")
        msg = (name, rank, text)
    r.end()
    return msg, generation


def decode(frame) -> Tuple:
    return decode_with_generation(frame)[0]
