"""Engine and request lifecycle (reference: contracts/lifecycle.mbt:1-66)."""
from __future__ import annotations

import enum

PROTOCOL_VERSION = "lunaflux.inference.v1alpha1"


class EngineState(enum.Enum):
    LOADING = "loading"
    WARMING = "warming"
    READY = "ready"
    DRAINING = "draining"
    STOPPED = "stopped"
    FAILED = "failed"


class RequestState(enum.Enum):
    ADMITTED = "admitted"
    TOKENIZING = "tokenizing"
    WAITING = "waiting"
    PREFILL = "prefill"
    DECODE = "decode"
    FINISHING = "finishing"
    CANCELLED = "cancelled"
    FINISHED = "finished"
    FAILED = "failed"

    @property
    def terminal(self) -> bool:
        return self in (RequestState.CANCELLED, RequestState.FINISHED, RequestState.FAILED)


_S = RequestState
# The v1 transition table; terminal states have no successors.
_TRANSITIONS = {
    _S.ADMITTED: {_S.TOKENIZING, _S.CANCELLED, _S.FAILED},
    _S.TOKENIZING: {_S.WAITING, _S.CANCELLED, _S.FAILED},
    _S.WAITING: {_S.PREFILL, _S.CANCELLED, _S.FAILED},
    _S.PREFILL: {_S.PREFILL, _S.DECODE, _S.FINISHING, _S.CANCELLED, _S.FAILED},
    _S.DECODE: {_S.DECODE, _S.FINISHING, _S.CANCELLED, _S.FAILED},
    _S.FINISHING: {_S.FINISHED, _S.CANCELLED, _S.FAILED},
    _S.CANCELLED: set(),
    _S.FINISHED: set(),
    _S.FAILED: set(),
}


def can_transition(current: RequestState, nxt: RequestState) -> bool:
    return nxt in _TRANSITIONS[current]
