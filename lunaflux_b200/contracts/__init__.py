"""Canonical request / event vocabulary and lifecycle state machines.

Mirrors the reference's `contracts` and `contracts/inference` packages
(contracts/lifecycle.mbt:1-66, contracts/inference/request.mbt,
contracts/inference/events.mbt:217-324, contracts/inference/limits.mbt:1-140,
contracts/inference/errors.mbt:7-50): the same states, transition table,
limits, validation categories and event kinds, as frozen Python dataclasses.
"""
from .lifecycle import EngineState, RequestState, PROTOCOL_VERSION, can_transition  # noqa: F401
from .inference import (  # noqa: F401
    ContractError, ContractField, ContractIssue, InferenceLimits, SamplingMode, SamplingParameters,
    StopConditions, GenerateRequest, CacheScope, FinishReason, PublicErrorCode, Usage,
    AcceptedEvent, TokenEvent, CompletedEvent, FailedEvent, StreamEvent, default_limits, derive_seed,
    RETRYABLE_CODES, validate_event,
)
