"""The inference contract: request validation categories and their fixed
precedence, hostile UTF-8, sampling canonical forms, limits, and stream-event
checks.  Every error is payload free: (field, issue, index), never bytes of
the request.

Modelled on the reference's contracts/inference tests (request_test.mbt,
request_authority_wbtest.mbt: "GenerateRequest adjacent validation
precedence is fixed", "GenerateRequest rejects noncanonical forged greedy
sampling", "sampling rejects non-finite and invalid filters", "stop
conditions reject duplicates IDs invalid UTF-8 and every bound", "canonical
request validates exact token context without overflow"; events_test.mbt:
"token event validates UTF-8 token identity and position bounds", "usage
construction and advancement enforce monotonic accounting", "terminal events
expose bounded reasons usage and retryability"; "UTF-8 validation rejects
every hostile class and accepts supplementary").
"""
import math

import pytest

from lunaflux_b200.contracts.inference import (HARD_MAX_CONTEXT_TOKENS, HARD_MAX_TEMPERATURE, RETRYABLE_CODES,
                                               CachePermission, CacheScope, CompletedEvent, ContractError,
                                               ContractField as F, ContractIssue as I, FailedEvent, FinishReason,
                                               GenerateRequest, InferenceLimits, PublicErrorCode, SamplingMode,
                                               SamplingParameters, StopConditions, TokenEvent, Usage, default_limits,
                                               validate_event)

LIM = default_limits(1000, 4096)

HOSTILE_UTF8 = {
    "overlong slash": b"\xc0\xaf",
    "overlong nul": b"\xe0\x80\x80",
    "surrogate": b"\xed\xa0\x80",
    "beyond U+10FFFF": b"\xf4\x90\x80\x80",
    "truncated 3-byte": b"\xe2\x82",
    "stray continuation": b"\x80",
    "5-byte form": b"\xf8\x88\x80\x80\x80",
    "invalid byte FF": b"a\xffb",
}
VALID_UTF8 = [b"plain", "é".encode(), "€".encode(), "😀".encode(), "\U0010ffff".encode(), b"\x00"]


def err(req_or_fn, limits=LIM):
    with pytest.raises(ContractError) as e:
        if callable(req_or_fn):
            req_or_fn()
        else:
            req_or_fn.validate(limits)
    assert "\\x" not in str(e.value) and "b'" not in str(e.value)       # no payload bytes in the message
    return e.value.field, e.value.issue, e.value.index


def req(**kw):
    base = dict(request_id=1, input_tokens=(1, 2, 3), max_new_tokens=4)
    base.update(kw)
    return GenerateRequest(**base)


# ----------------------------------------------------------------------------- inputs
def test_input_shapes():
    assert err(req(input_tokens=None)) == (F.INPUT_TOKEN, I.INCONSISTENT, 0)
    assert err(req(input_text=b"x")) == (F.INPUT_TOKEN, I.INCONSISTENT, 0)
    assert err(req(input_tokens=())) == (F.INPUT_TOKEN, I.EMPTY, 0)
    assert err(req(input_tokens=tuple(range(1, 4098)))) == (F.INPUT_TOKEN, I.TOO_MANY, 0)
    assert err(req(input_tokens=(1, 2, 1000, 5))) == (F.INPUT_TOKEN, I.OUT_OF_RANGE, 2)
    assert err(req(input_tokens=(1, -1))) == (F.INPUT_TOKEN, I.OUT_OF_RANGE, 1)
    req(input_tokens=(0, 999)).validate(LIM)                       # both ends of the vocabulary
    assert err(req(input_tokens=None, input_text=b"")) == (F.INPUT_TEXT, I.EMPTY, 0)
    lim = InferenceLimits(8, 64, 16, 64, 999, max_top_k=64)
    assert err(req(input_tokens=None, input_text=b"123456789"), lim) == (F.INPUT_TEXT, I.TOO_LONG, 0)
    req(input_tokens=None, input_text=b"12345678").validate(lim)


@pytest.mark.parametrize("name", sorted(HOSTILE_UTF8))
def test_hostile_utf8_is_rejected_in_text_and_stop_strings(name):
    bad = HOSTILE_UTF8[name]
    assert err(req(input_tokens=None, input_text=bad)) == (F.INPUT_TEXT, I.INVALID_FORMAT, 0)
    stop = StopConditions((), (b"ok", bad))
    assert err(req(stop=stop)) == (F.STOP_STRING, I.INVALID_FORMAT, 1)


def test_valid_utf8_including_supplementary_planes_is_accepted():
    for s in VALID_UTF8:
        req(input_tokens=None, input_text=s).validate(LIM)
        req(stop=StopConditions((), (s,))).validate(LIM)


def test_request_id_range():
    assert err(req(request_id=-1)) == (F.REQUEST_ID, I.OUT_OF_RANGE, 0)
    assert err(req(request_id=1 << 64)) == (F.REQUEST_ID, I.OUT_OF_RANGE, 0)
    req(request_id=(1 << 64) - 1).validate(LIM)
    req(request_id=0).validate(LIM)


# ----------------------------------------------------------------------------- context
def test_max_new_tokens_and_context_ceiling():
    assert err(req(max_new_tokens=0)) == (F.MAXIMUM_NEW_TOKENS, I.OUT_OF_RANGE, 0)
    assert err(req(max_new_tokens=4097)) == (F.MAXIMUM_NEW_TOKENS, I.OUT_OF_RANGE, 0)
    assert err(req(context_ceiling=0)) == (F.CONTEXT_CEILING, I.OUT_OF_RANGE, 0)
    assert err(req(context_ceiling=4097)) == (F.CONTEXT_CEILING, I.OUT_OF_RANGE, 0)
    assert err(req(max_new_tokens=9, context_ceiling=8)) == (F.CONTEXT_CEILING, I.INCONSISTENT, 0)
    # prompt + every requested token must fit: exactly fitting is fine, one more is not
    req(input_tokens=(1, 2, 3), max_new_tokens=5, context_ceiling=8).validate(LIM)
    assert err(req(input_tokens=(1, 2, 3, 4), max_new_tokens=5, context_ceiling=8)) == \
        (F.CONTEXT_CEILING, I.INCONSISTENT, 0)
    # a text prompt is measured once it is tokenized (by the service)
    req(input_tokens=None, input_text=b"a" * 100, max_new_tokens=5, context_ceiling=8).validate(LIM)


# ----------------------------------------------------------------------------- sampling
def test_greedy_must_be_canonical():
    g = SamplingMode.GREEDY
    assert err(req(sampling=SamplingParameters(g, 0.5, 1, 0.5))) == (F.TEMPERATURE, I.INCONSISTENT, 0)
    assert err(req(sampling=SamplingParameters(g, 1.0, 1, 0.5))) == (F.TOP_K, I.INCONSISTENT, 0)
    assert err(req(sampling=SamplingParameters(g, 1.0, None, 0.5))) == (F.TOP_P, I.INCONSISTENT, 0)
    req(sampling=SamplingParameters.greedy()).validate(LIM)


@pytest.mark.parametrize("value", [math.nan, math.inf, -math.inf])
def test_sampling_rejects_non_finite_values(value):
    assert err(req(sampling=SamplingParameters.sample(value))) == (F.TEMPERATURE, I.NON_FINITE, 0)
    assert err(req(sampling=SamplingParameters.sample(0.7, top_p=value))) == (F.TOP_P, I.NON_FINITE, 0)


def test_sampling_bounds():
    s = SamplingParameters.sample
    for t in (0.0, -1.0, LIM.max_temperature * 1.0001):
        assert err(req(sampling=s(t))) == (F.TEMPERATURE, I.OUT_OF_RANGE, 0)
    req(sampling=s(LIM.max_temperature)).validate(LIM)
    for k in (0, -3, LIM.max_top_k + 1):
        assert err(req(sampling=s(0.7, top_k=k))) == (F.TOP_K, I.OUT_OF_RANGE, 0)
    req(sampling=s(0.7, top_k=LIM.max_top_k)).validate(LIM)
    for p in (0.0, -0.1, 1.0000001):
        assert err(req(sampling=s(0.7, top_p=p))) == (F.TOP_P, I.OUT_OF_RANGE, 0)
    req(sampling=s(0.7, top_p=1.0)).validate(LIM)
    for seed in (0, -1, 1 << 64):
        assert err(req(sampling=s(0.7, seed=seed))) == (F.SAMPLING_SEED, I.OUT_OF_RANGE, 0)
    req(sampling=s(0.7, seed=(1 << 64) - 1)).validate(LIM)


# ----------------------------------------------------------------------------- stops, cache, trace, deadline
def test_stop_conditions_every_bound():
    lim = InferenceLimits(64, 64, 16, 64, 999, max_stop_token_ids=3, max_stop_strings=2, max_stop_string_bytes=4,
                          max_top_k=64)
    st = StopConditions
    assert err(req(stop=st((1, 2, 3, 4))), lim) == (F.STOP_TOKEN, I.TOO_MANY, 0)
    assert err(req(stop=st((1, 1000))), lim) == (F.STOP_TOKEN, I.OUT_OF_RANGE, 1)
    assert err(req(stop=st((5, 6, 5))), lim) == (F.STOP_TOKEN, I.DUPLICATE, 2)
    assert err(req(stop=st((), (b"a", b"b", b"c"))), lim) == (F.STOP_STRING, I.TOO_MANY, 0)
    assert err(req(stop=st((), (b"a", b""))), lim) == (F.STOP_STRING, I.EMPTY, 1)
    assert err(req(stop=st((), (b"abcde",))), lim) == (F.STOP_STRING, I.TOO_LONG, 0)
    assert err(req(stop=st((), (b"ab", b"ab"))), lim) == (F.STOP_STRING, I.DUPLICATE, 1)
    req(stop=st((1, 2, 3), (b"abcd", b"e"))).validate(lim)


def test_cache_scope_trace_and_deadline():
    assert err(req(cache=CacheScope(b"tenant 1"))) == (F.CACHE_SCOPE, I.INVALID_FORMAT, 6)
    assert err(req(cache=CacheScope(b"a" * (LIM.max_cache_scope_bytes + 1)))) == (F.CACHE_SCOPE, I.TOO_LONG, 0)
    for scope in (b"", b"tenant-1", b"A.b_c:9"):
        req(cache=CacheScope(scope, CachePermission.READ_ONLY)).validate(LIM)
    assert err(req(trace=b"t" * (LIM.max_trace_bytes + 1))) == (F.TRACE_CORRELATION, I.TOO_LONG, 0)
    req(trace=b"t" * LIM.max_trace_bytes).validate(LIM)
    assert err(req(deadline_millis=0)) == (F.DEADLINE_BUDGET, I.OUT_OF_RANGE, 0)
    assert err(req(deadline_millis=LIM.max_deadline_millis + 1)) == (F.DEADLINE_BUDGET, I.OUT_OF_RANGE, 0)
    req(deadline_millis=LIM.max_deadline_millis).validate(LIM)


def test_validation_precedence_is_fixed():
    """A request with every fault reports them one at a time, in a fixed
    order, as each earlier one is repaired."""
    faults = [
        ("request_id", -1, F.REQUEST_ID),
        ("input_tokens", (), F.INPUT_TOKEN),
        ("max_new_tokens", 0, F.MAXIMUM_NEW_TOKENS),
        ("context_ceiling", 0, F.CONTEXT_CEILING),
        ("sampling", SamplingParameters(SamplingMode.GREEDY, 2.0), F.TEMPERATURE),
        ("stop", StopConditions((1, 1)), F.STOP_TOKEN),
        ("deadline_millis", 0, F.DEADLINE_BUDGET),
        ("cache", CacheScope(b"no spaces"), F.CACHE_SCOPE),
        ("trace", b"t" * 1000, F.TRACE_CORRELATION),
    ]
    good = req()
    bad = {k: v for k, v, _ in faults}
    for i, (_, _, field) in enumerate(faults):
        fields = {**good.__dict__, **{k: v for k, v, _ in faults[i:]}}
        assert err(GenerateRequest(**fields))[0] is field, (i, field)
    assert len(bad) == len(faults)
    GenerateRequest(**good.__dict__).validate(LIM)


# ----------------------------------------------------------------------------- limits
def test_forged_limits_are_rejected():
    base = dict(max_text_bytes=64, max_input_tokens=64, max_new_tokens=16, max_context_tokens=64, max_token_id=999,
                max_top_k=64)
    InferenceLimits(**base)
    bad = [dict(max_text_bytes=0), dict(max_input_tokens=65), dict(max_new_tokens=65),
           dict(max_context_tokens=HARD_MAX_CONTEXT_TOKENS + 1), dict(max_token_id=-1),
           dict(max_stop_token_ids=0), dict(max_top_k=1001), dict(max_temperature=math.nan),
           dict(max_temperature=HARD_MAX_TEMPERATURE * 2), dict(max_deadline_millis=0)]
    for b in bad:
        assert err(lambda: InferenceLimits(**{**base, **b})) == (F.LIMIT, I.OUT_OF_RANGE, 0), b


# ----------------------------------------------------------------------------- events
def test_token_event_bounds_and_utf8():
    validate_event(TokenEvent(1, 0, 0, b""))
    validate_event(TokenEvent(1, 5, 999, "é😀".encode()), max_token_id=999)
    assert err(lambda: validate_event(TokenEvent(1, -1, 3))) == (F.TOKEN_POSITION, I.OUT_OF_RANGE, 0)
    assert err(lambda: validate_event(TokenEvent(1, 0, 1000), max_token_id=999)) == \
        (F.INPUT_TOKEN, I.OUT_OF_RANGE, 0)
    for name, bad in HOSTILE_UTF8.items():
        assert err(lambda: validate_event(TokenEvent(1, 0, 3, bad))) == (F.DECODED_DELTA, I.INVALID_FORMAT, 0), name
    assert err(lambda: validate_event(TokenEvent(1, 0, 3, b"a" * 9), max_delta_bytes=8)) == \
        (F.DECODED_DELTA, I.TOO_LONG, 0)
    assert err(lambda: validate_event(TokenEvent(-1, 0, 3))) == (F.REQUEST_ID, I.OUT_OF_RANGE, 0)


def test_usage_accounting_is_consistent():
    validate_event(Usage(10, 10, 0))
    assert err(lambda: validate_event(Usage(10, 11, 0))) == (F.USAGE, I.INCONSISTENT, 0)
    for u in (Usage(-1, 0, 0), Usage(1, 0, -1), Usage(HARD_MAX_CONTEXT_TOKENS + 1, 0, 0)):
        assert err(lambda: validate_event(u)) == (F.USAGE, I.OUT_OF_RANGE, 0)
    assert Usage(7, 3, 5).total_tokens == 12


def test_terminal_events_reasons_usage_and_retryability():
    for reason in FinishReason:
        validate_event(CompletedEvent(1, reason, Usage(3, 0, 2), "ü".encode()))
    assert err(lambda: validate_event(CompletedEvent(1, FinishReason.TOKEN_LIMIT, Usage(3, 4, 2)))) == \
        (F.USAGE, I.INCONSISTENT, 0)
    assert err(lambda: validate_event(CompletedEvent(1, FinishReason.TOKEN_LIMIT, Usage(3, 0, 2), b"\xc3"))) == \
        (F.DECODED_DELTA, I.INVALID_FORMAT, 0)
    assert RETRYABLE_CODES == {PublicErrorCode.OVERLOADED, PublicErrorCode.WORKER_UNAVAILABLE}
    for code in PublicErrorCode:
        validate_event(FailedEvent(1, code, code in RETRYABLE_CODES))
        assert err(lambda: validate_event(FailedEvent(1, code, code not in RETRYABLE_CODES))) == \
            (F.PUBLIC_ERROR_CODE, I.INCONSISTENT, 0)


def test_encoder_refuses_an_event_that_breaks_the_contract():
    from lunaflux_b200.service.framed_wire import FramedWireError, encode_event
    encode_event(TokenEvent(1, 4, 7, b"ok"))
    with pytest.raises(FramedWireError):
        encode_event(TokenEvent(1, 4, 7, b"\xff"))
    with pytest.raises(FramedWireError):
        encode_event(FailedEvent(1, PublicErrorCode.INTERNAL, True))
