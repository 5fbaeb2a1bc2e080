"""The strict configuration document (reference: config/document tests:
"malformed JSON and non-object roots fail closed", "nested and
escaped-equivalent duplicate fields fail before core parsing", "unknown and
missing fields fail", "wrong types and non-integral numbers are rejected",
"focused integer ranges are enforced during construction", "byte limits and
invalid UTF-8 are rejected before JSON parsing"; config/runtime_resolved:
"identical validated inputs resolve identically")."""
import json

import pytest

from lunaflux_b200.config.records import MAX_DOCUMENT_BYTES, ConfigError, parse_document, resolve

BASE = {"schema_version": 1, "model": {"preset": "llama3-8b"}}


def doc(**sections):
    d = json.loads(json.dumps(BASE))
    for k, v in sections.items():
        d[k] = {**d.get(k, {}), **v}
    return json.dumps(d)


def test_minimal_document_and_defaults():
    cfg = parse_document(json.dumps(BASE))
    assert cfg.model.preset == "llama3-8b" and cfg.parallel.tp == 1 and cfg.kernels.use_graphs


@pytest.mark.parametrize("text", [b"", b"{", b"[1]", b"null", b'"x"', b"\xff{}",
                                  b'{"schema_version": 1, "model": {"preset": "a", "pr\\u0065set": "b"}}',
                                  b'{"schema_version": 1, "model": {"preset": "a"}, "model": {"preset": "b"}}'])
def test_malformed_documents_fail_closed(text):
    with pytest.raises(ConfigError):
        parse_document(text)


def test_byte_limit_is_checked_before_parsing():
    big = doc(model={"artifact_path": "a" * MAX_DOCUMENT_BYTES})
    with pytest.raises(ConfigError, match="exceeds"):
        parse_document(big)


@pytest.mark.parametrize("section,fields", [
    ("service", {"listen_host": 5}), ("service", {"diagnostic_mode": 1}), ("service", {"listen_port": 80.0}),
    ("model", {"preset": 7}), ("model", {"seed": 1.5}), ("model", {"artifact_path": 3}),
    ("model", {"architecture_allowlist": [1]}), ("device", {"visible_devices": ["a"]}),
    ("cache", {"prefix_enabled": "yes"}), ("kernels", {"use_graphs": 1}), ("scheduler", {"max_active_requests": True}),
    ("scheduler", {"step_token_budget": "8192"}), ("parallel", {"tp": 2.0}),
])
def test_wrong_types_are_rejected(section, fields):
    with pytest.raises(ConfigError, match="wrong type"):
        parse_document(doc(**{section: fields}))


@pytest.mark.parametrize("section,fields", [
    ("model", {"seed": -1}), ("device", {"visible_devices": [-1]}), ("device", {"visible_devices": [0, 0]}),
    ("kernels", {"graph_batch_sizes": [0]}), ("kernels", {"graph_batch_sizes": [2, 1]}),
    ("scheduler", {"max_active_requests": 0}), ("scheduler", {"prefill_chunk_tokens": 10 ** 9}),
    ("service", {"listen_port": 70000}), ("cache", {"tokens_per_page": 32}), ("parallel", {"tp": 3}),
    ("model", {"expected_digest": "ABC"}),
])
def test_ranges_are_enforced(section, fields):
    with pytest.raises(ConfigError):
        parse_document(doc(**{section: fields}))


def test_unknown_and_missing_fields():
    for bad in [dict(BASE, extra={}), dict(BASE, schema_version=2), {"schema_version": 1},
                {**BASE, "model": {"preset": "x", "bogus": 1}}, {**BASE, "model": {}}]:
        with pytest.raises(ConfigError):
            parse_document(json.dumps(bad))


def test_identical_inputs_resolve_identically():
    a = resolve(parse_document(doc(scheduler={"max_active_requests": 32})), 2 << 20, free_bytes=8 << 30,
                max_context=4096)
    b = resolve(parse_document(doc(scheduler={"max_active_requests": 32})), 2 << 20, free_bytes=8 << 30,
                max_context=4096)
    assert a == b and a.max_rows == 32 and all(x <= 32 for x in a.graph_batch_sizes)
