"""Transport-independent generation request and streaming events.

Reference: contracts/inference/request.mbt:3-361, events.mbt:3-324,
sampling.mbt, sampling_seed.mbt, limits.mbt:1-140, errors.mbt:7-50.
Validation errors carry only a bounded field, an issue category and a
collection index, never payload bytes (docs/PRODUCT_CONTRACT.md:86-90).
"""
from __future__ import annotations

import dataclasses
import enum
import math
from typing import Optional, Sequence, Tuple, Union


class ContractField(enum.Enum):
    PROTOCOL_VERSION = 0
    REQUEST_ID = 1
    REQUEST_GENERATION = 2
    LIMIT = 3
    INPUT_TOKEN = 4
    INPUT_TEXT = 5
    MAXIMUM_NEW_TOKENS = 8
    CONTEXT_CEILING = 9
    TEMPERATURE = 10
    TOP_K = 11
    TOP_P = 12
    SAMPLING_SEED = 13
    STOP_TOKEN = 14
    STOP_STRING = 15
    DEADLINE_BUDGET = 16
    CACHE_SCOPE = 17
    TRACE_CORRELATION = 18
    DECODED_DELTA = 19
    TOKEN_POSITION = 20
    USAGE = 21
    PUBLIC_ERROR_CODE = 24


class ContractIssue(enum.Enum):
    EMPTY = 0
    TOO_LONG = 1
    TOO_MANY = 2
    INVALID_FORMAT = 3
    OUT_OF_RANGE = 4
    DUPLICATE = 5
    NON_FINITE = 6
    NOT_MONOTONIC = 7
    INCONSISTENT = 8
    UNSUPPORTED = 9


class ContractError(ValueError):
    """Payload-free validation error: (field, issue, index)."""

    def __init__(self, field: ContractField, issue: ContractIssue, index: int = 0):
        super().__init__(f"{field.name}:{issue.name}:{index}")
        self.field = field
        self.issue = issue
        self.index = index


def _bad(field, issue, index=0):
    raise ContractError(field, issue, index)


HARD_MAX_TEXT_BYTES = 1048576
HARD_MAX_INPUT_TOKENS = 262144
HARD_MAX_NEW_TOKENS = 65536
HARD_MAX_CONTEXT_TOKENS = 262144
HARD_MAX_TOKEN_ID = 16777215
HARD_MAX_STOP_TOKEN_IDS = 256
HARD_MAX_STOP_STRINGS = 64
HARD_MAX_STOP_STRING_BYTES = 4096
HARD_MAX_TRACE_BYTES = 256
HARD_MAX_CACHE_SCOPE_BYTES = 256
HARD_MAX_DECODED_DELTA_BYTES = 16384
HARD_MAX_DEADLINE_MILLIS = 86400000
HARD_MAX_TOP_K = 1048576
HARD_MAX_TEMPERATURE = 100.0


@dataclasses.dataclass(frozen=True)
class InferenceLimits:
    max_text_bytes: int
    max_input_tokens: int
    max_new_tokens: int
    max_context_tokens: int
    max_token_id: int
    max_stop_token_ids: int = 64
    max_stop_strings: int = 16
    max_stop_string_bytes: int = 256
    max_trace_bytes: int = 128
    max_cache_scope_bytes: int = 128
    max_decoded_delta_bytes: int = 4096
    max_deadline_millis: int = 3600000
    max_top_k: int = 1024
    max_temperature: float = 10.0

    def __post_init__(self):
        def pb(v, m):
            return 0 < v <= m

        ok = (pb(self.max_text_bytes, HARD_MAX_TEXT_BYTES) and pb(self.max_input_tokens, HARD_MAX_INPUT_TOKENS)
              and pb(self.max_new_tokens, HARD_MAX_NEW_TOKENS)
              and pb(self.max_context_tokens, HARD_MAX_CONTEXT_TOKENS)
              and self.max_input_tokens <= self.max_context_tokens
              and self.max_new_tokens <= self.max_context_tokens
              and 0 <= self.max_token_id <= HARD_MAX_TOKEN_ID
              and pb(self.max_stop_token_ids, HARD_MAX_STOP_TOKEN_IDS)
              and pb(self.max_stop_strings, HARD_MAX_STOP_STRINGS)
              and pb(self.max_stop_string_bytes, HARD_MAX_STOP_STRING_BYTES)
              and pb(self.max_trace_bytes, HARD_MAX_TRACE_BYTES)
              and pb(self.max_cache_scope_bytes, HARD_MAX_CACHE_SCOPE_BYTES)
              and pb(self.max_decoded_delta_bytes, HARD_MAX_DECODED_DELTA_BYTES)
              and 0 < self.max_deadline_millis <= HARD_MAX_DEADLINE_MILLIS
              and pb(self.max_top_k, HARD_MAX_TOP_K) and self.max_top_k <= self.max_token_id + 1
              and math.isfinite(self.max_temperature) and 0.0 < self.max_temperature <= HARD_MAX_TEMPERATURE)
        if not ok:
            _bad(ContractField.LIMIT, ContractIssue.OUT_OF_RANGE)


def default_limits(vocab_size: int, max_context: int) -> InferenceLimits:
    return InferenceLimits(max_text_bytes=1 << 20, max_input_tokens=max_context, max_new_tokens=min(max_context, 65536),
                           max_context_tokens=max_context, max_token_id=vocab_size - 1,
                           max_top_k=min(1024, vocab_size))


class SamplingMode(enum.Enum):
    GREEDY = 0
    SAMPLE = 1


@dataclasses.dataclass(frozen=True)
class SamplingParameters:
    """Greedy, or temperature / top-k / top-p sampling with a non-zero seed.

    reference: contracts/inference/sampling.mbt (temperature <= max, top_k <=
    max, top_p in (0, 1]) and sampling_seed.mbt (seed != 0).
    """
    mode: SamplingMode = SamplingMode.GREEDY
    temperature: float = 1.0
    top_k: Optional[int] = None
    top_p: Optional[float] = None
    seed: int = 1

    def validate(self, limits: InferenceLimits) -> "SamplingParameters":
        if self.mode is SamplingMode.GREEDY:
            # greedy carries the neutral values only: a filter or temperature
            # that would be ignored is a client error, not a silent no-op
            # (reference: request_authority_wbtest.mbt:310-324)
            if self.temperature != 1.0:
                _bad(ContractField.TEMPERATURE, ContractIssue.INCONSISTENT)
            if self.top_k is not None:
                _bad(ContractField.TOP_K, ContractIssue.INCONSISTENT)
            if self.top_p is not None:
                _bad(ContractField.TOP_P, ContractIssue.INCONSISTENT)
        elif self.mode is SamplingMode.SAMPLE:
            if not math.isfinite(self.temperature):
                _bad(ContractField.TEMPERATURE, ContractIssue.NON_FINITE)
            if not (0.0 < self.temperature <= limits.max_temperature):
                _bad(ContractField.TEMPERATURE, ContractIssue.OUT_OF_RANGE)
            if self.top_k is not None and not (0 < self.top_k <= limits.max_top_k):
                _bad(ContractField.TOP_K, ContractIssue.OUT_OF_RANGE)
            if self.top_p is not None:
                if not math.isfinite(self.top_p):
                    _bad(ContractField.TOP_P, ContractIssue.NON_FINITE)
                if not (0.0 < self.top_p <= 1.0):
                    _bad(ContractField.TOP_P, ContractIssue.OUT_OF_RANGE)
        if not (0 < self.seed < (1 << 64)):
            _bad(ContractField.SAMPLING_SEED, ContractIssue.OUT_OF_RANGE)
        return self

    @staticmethod
    def greedy() -> "SamplingParameters":
        return SamplingParameters()

    @staticmethod
    def sample(temperature: float, top_k: Optional[int] = None, top_p: Optional[float] = None,
               seed: int = 1) -> "SamplingParameters":
        return SamplingParameters(SamplingMode.SAMPLE, temperature, top_k, top_p, seed)


def derive_seed(global_seed: int, request_index: int) -> int:
    """Non-zero per-request seed derived from a global seed (which may be 0).

    splitmix64 finaliser of (global_seed, index); a zero result maps to the
    golden-ratio constant, as the reference's counter_state does
    (sampling/rng.mbt).
    """
    m = (1 << 64) - 1
    v = (global_seed + (request_index + 1) * 0x9E3779B97F4A7C15) & m
    v = ((v ^ (v >> 30)) * 0xBF58476D1CE4E5B9) & m
    v = ((v ^ (v >> 27)) * 0x94D049BB133111EB) & m
    v ^= v >> 31
    return v if v != 0 else 0x9E3779B97F4A7C15


@dataclasses.dataclass(frozen=True)
class StopConditions:
    token_ids: Tuple[int, ...] = ()
    strings: Tuple[bytes, ...] = ()

    def validate(self, limits: InferenceLimits) -> "StopConditions":
        if len(self.token_ids) > limits.max_stop_token_ids:
            _bad(ContractField.STOP_TOKEN, ContractIssue.TOO_MANY)
        seen = set()
        for i, t in enumerate(self.token_ids):
            if not (0 <= t <= limits.max_token_id):
                _bad(ContractField.STOP_TOKEN, ContractIssue.OUT_OF_RANGE, i)
            if t in seen:
                _bad(ContractField.STOP_TOKEN, ContractIssue.DUPLICATE, i)
            seen.add(t)
        if len(self.strings) > limits.max_stop_strings:
            _bad(ContractField.STOP_STRING, ContractIssue.TOO_MANY)
        sseen = set()
        for i, s in enumerate(self.strings):
            if not s:
                _bad(ContractField.STOP_STRING, ContractIssue.EMPTY, i)
            if len(s) > limits.max_stop_string_bytes:
                _bad(ContractField.STOP_STRING, ContractIssue.TOO_LONG, i)
            try:
                s.decode("utf-8")
            except UnicodeDecodeError:
                _bad(ContractField.STOP_STRING, ContractIssue.INVALID_FORMAT, i)
            if s in sseen:
                _bad(ContractField.STOP_STRING, ContractIssue.DUPLICATE, i)
            sseen.add(s)
        return self


class CachePermission(enum.Enum):
    """Prefix-cache permission; the values are the framed-wire codes."""
    DISABLED = 0
    READ_ONLY = 1
    READ_WRITE = 2


@dataclasses.dataclass(frozen=True)
class CacheScope:
    """Prefix-cache partition.  Entries are only shared inside one scope."""
    scope: bytes = b""
    permission: CachePermission = CachePermission.READ_WRITE

    def validate(self, limits: InferenceLimits) -> "CacheScope":
        if len(self.scope) > limits.max_cache_scope_bytes:
            _bad(ContractField.CACHE_SCOPE, ContractIssue.TOO_LONG)
        for i, b in enumerate(self.scope):
            if not (48 <= b <= 57 or 65 <= b <= 90 or 97 <= b <= 122 or b in b"-_.:"):
                _bad(ContractField.CACHE_SCOPE, ContractIssue.INVALID_FORMAT, i)
        return self


@dataclasses.dataclass(frozen=True)
class GenerateRequest:
    """One validated generation request (token or text input)."""
    request_id: int
    input_tokens: Optional[Tuple[int, ...]] = None
    input_text: Optional[bytes] = None
    max_new_tokens: int = 16
    context_ceiling: Optional[int] = None
    sampling: SamplingParameters = SamplingParameters()
    stop: StopConditions = StopConditions()
    streaming: bool = True
    deadline_millis: Optional[int] = None
    cache: CacheScope = CacheScope()
    trace: Optional[bytes] = None
    # loaded-model identity the client targets (lowercase SHA-256 hex, "" = any)
    model_content_digest: str = ""
    model_plan_digest: str = ""

    def validate(self, limits: InferenceLimits) -> "GenerateRequest":
        if not (0 <= self.request_id < (1 << 64)):
            _bad(ContractField.REQUEST_ID, ContractIssue.OUT_OF_RANGE)
        if (self.input_tokens is None) == (self.input_text is None):
            _bad(ContractField.INPUT_TOKEN, ContractIssue.INCONSISTENT)
        if self.input_tokens is not None:
            if len(self.input_tokens) == 0:
                _bad(ContractField.INPUT_TOKEN, ContractIssue.EMPTY)
            if len(self.input_tokens) > limits.max_input_tokens:
                _bad(ContractField.INPUT_TOKEN, ContractIssue.TOO_MANY)
            for i, t in enumerate(self.input_tokens):
                if not (0 <= t <= limits.max_token_id):
                    _bad(ContractField.INPUT_TOKEN, ContractIssue.OUT_OF_RANGE, i)
        else:
            if len(self.input_text) == 0:
                _bad(ContractField.INPUT_TEXT, ContractIssue.EMPTY)
            if len(self.input_text) > limits.max_text_bytes:
                _bad(ContractField.INPUT_TEXT, ContractIssue.TOO_LONG)
            try:
                self.input_text.decode("utf-8")
            except UnicodeDecodeError:
                _bad(ContractField.INPUT_TEXT, ContractIssue.INVALID_FORMAT)
        if not (0 < self.max_new_tokens <= limits.max_new_tokens):
            _bad(ContractField.MAXIMUM_NEW_TOKENS, ContractIssue.OUT_OF_RANGE)
        if self.context_ceiling is not None:
            # reference: contracts/inference/request.mbt:272-281 (the prompt and
            # every requested token must fit under the ceiling)
            if not (0 < self.context_ceiling <= limits.max_context_tokens):
                _bad(ContractField.CONTEXT_CEILING, ContractIssue.OUT_OF_RANGE)
            if self.max_new_tokens > self.context_ceiling:
                _bad(ContractField.CONTEXT_CEILING, ContractIssue.INCONSISTENT)
            if (self.input_tokens is not None
                    and len(self.input_tokens) > self.context_ceiling - self.max_new_tokens):
                _bad(ContractField.CONTEXT_CEILING, ContractIssue.INCONSISTENT)
        self.sampling.validate(limits)
        self.stop.validate(limits)
        if self.deadline_millis is not None and not (0 < self.deadline_millis <= limits.max_deadline_millis):
            _bad(ContractField.DEADLINE_BUDGET, ContractIssue.OUT_OF_RANGE)
        self.cache.validate(limits)
        if self.trace is not None and len(self.trace) > limits.max_trace_bytes:
            _bad(ContractField.TRACE_CORRELATION, ContractIssue.TOO_LONG)
        return self


# ---------------------------------------------------------------------------
# Events (events.mbt:217-324)
# ---------------------------------------------------------------------------
class FinishReason(enum.Enum):
    STOP_SEQUENCE = 1
    TOKEN_LIMIT = 2
    CANCELLED = 3


class PublicErrorCode(enum.Enum):
    """Bounded machine-readable failure codes; the value is the wire string."""
    INVALID_REQUEST = "invalid_request"
    OVERLOADED = "overloaded"
    DEADLINE_EXCEEDED = "deadline_exceeded"
    WORKER_UNAVAILABLE = "worker_unavailable"
    INTERNAL = "internal"
    CONTEXT_OVERFLOW = "context_overflow"
    CANCELLED = "cancelled"


@dataclasses.dataclass(frozen=True)
class Usage:
    input_tokens: int
    cached_input_tokens: int
    output_tokens: int

    @property
    def total_tokens(self) -> int:
        return self.input_tokens + self.output_tokens


@dataclasses.dataclass(frozen=True)
class AcceptedEvent:
    request_id: int


@dataclasses.dataclass(frozen=True)
class TokenEvent:
    request_id: int
    position: int
    token_id: int
    delta: bytes = b""


@dataclasses.dataclass(frozen=True)
class CompletedEvent:
    request_id: int
    reason: FinishReason
    usage: Usage
    final_delta: bytes = b""


@dataclasses.dataclass(frozen=True)
class FailedEvent:
    request_id: int
    code: PublicErrorCode
    retryable: bool


StreamEvent = Union[AcceptedEvent, TokenEvent, CompletedEvent, FailedEvent, Usage]

# Failures a client may retry unchanged: the service was busy or lost a worker.
RETRYABLE_CODES = frozenset({PublicErrorCode.OVERLOADED, PublicErrorCode.WORKER_UNAVAILABLE})


def _utf8(data: bytes, field: ContractField, max_bytes: int):
    if len(data) > max_bytes:
        _bad(field, ContractIssue.TOO_LONG)
    try:
        data.decode("utf-8")
    except UnicodeDecodeError:
        _bad(field, ContractIssue.INVALID_FORMAT)


def validate_event(ev, max_token_id: int = HARD_MAX_TOKEN_ID,
                   max_delta_bytes: int = HARD_MAX_DECODED_DELTA_BYTES):
    """Checks an outgoing stream event: ids and positions in range, decoded
    text valid UTF-8 and bounded, usage counts consistent (cached input within
    the input), and a failure's retryability matching its code.  Reference:
    contracts/inference/events.mbt:3-324 and events_test.mbt ("token event
    validates UTF-8 token identity and position bounds", "usage construction
    and advancement enforce monotonic accounting", "terminal events expose
    bounded reasons usage and retryability")."""
    if isinstance(ev, Usage):        # the usage event belongs to the stream it is written on
        _validate_usage(ev)
        return ev
    if not (0 <= ev.request_id < (1 << 64)):
        _bad(ContractField.REQUEST_ID, ContractIssue.OUT_OF_RANGE)
    if isinstance(ev, TokenEvent):
        if not (0 <= ev.token_id <= max_token_id):
            _bad(ContractField.INPUT_TOKEN, ContractIssue.OUT_OF_RANGE)
        if not (0 <= ev.position < HARD_MAX_CONTEXT_TOKENS):
            _bad(ContractField.TOKEN_POSITION, ContractIssue.OUT_OF_RANGE)
        _utf8(ev.delta, ContractField.DECODED_DELTA, max_delta_bytes)
    elif isinstance(ev, CompletedEvent):
        if not isinstance(ev.reason, FinishReason):
            _bad(ContractField.PUBLIC_ERROR_CODE, ContractIssue.UNSUPPORTED)
        _validate_usage(ev.usage)
        _utf8(ev.final_delta, ContractField.DECODED_DELTA, max_delta_bytes)
    elif isinstance(ev, FailedEvent):
        if not isinstance(ev.code, PublicErrorCode):
            _bad(ContractField.PUBLIC_ERROR_CODE, ContractIssue.UNSUPPORTED)
        if bool(ev.retryable) != (ev.code in RETRYABLE_CODES):
            _bad(ContractField.PUBLIC_ERROR_CODE, ContractIssue.INCONSISTENT)
    return ev


def _validate_usage(u: Usage):
    for v in (u.input_tokens, u.cached_input_tokens, u.output_tokens):
        if not (0 <= v <= HARD_MAX_CONTEXT_TOKENS):
            _bad(ContractField.USAGE, ContractIssue.OUT_OF_RANGE)
    if u.cached_input_tokens > u.input_tokens:
        _bad(ContractField.USAGE, ContractIssue.INCONSISTENT)


def token_tuple(tokens: Sequence[int]) -> Tuple[int, ...]:
    return tuple(int(t) for t in tokens)
