"""Strict JSON: duplicate keys (also escape-equivalent ones) and NaN/Infinity
literals are rejected, nesting depth is bounded.

Reference: internal/json_guard/guard.mbt:18 (reject_duplicate_object_keys).
Python's decoder already unescapes keys before the hook sees them, so two
spellings of the same key collide here exactly as in the reference.
"""
from __future__ import annotations

import json
from typing import Any

MAX_DEPTH = 64


class StrictJsonError(ValueError):
    pass


def _pairs(pairs):
    out = {}
    for k, v in pairs:
        if k in out:
            raise StrictJsonError("duplicate object key")
        out[k] = v
    return out


def _reject_constant(name):
    raise StrictJsonError(f"non-finite literal {name} is not JSON")


def _depth(s: str) -> int:
    depth = best = 0
    in_str = esc = False
    for ch in s:
        if in_str:
            if esc:
                esc = False
            elif ch == "\\":
                esc = True
            elif ch == '"':
                in_str = False
        elif ch == '"':
            in_str = True
        elif ch in "[{":
            depth += 1
            best = max(best, depth)
        elif ch in "]}":
            depth -= 1
    return best


def loads_strict(text: str | bytes, max_depth: int = MAX_DEPTH) -> Any:
    if isinstance(text, (bytes, bytearray)):
        text = bytes(text).decode("utf-8")
    if _depth(text) > max_depth:
        raise StrictJsonError("JSON nesting too deep")
    return json.loads(text, object_pairs_hook=_pairs, parse_constant=_reject_constant)
