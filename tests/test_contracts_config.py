"""Contracts, strict JSON, configuration documents, safetensors and model specs (CPU)."""
import json
import struct

import pytest
import torch

from lunaflux_b200.config import ConfigError, parse_document, resolve
from lunaflux_b200.contracts import (ContractError, ContractField, ContractIssue, GenerateRequest, RequestState,
                                     SamplingParameters, StopConditions, can_transition, default_limits, derive_seed)
from lunaflux_b200.models.safetensors import SafetensorsError, SafetensorsFile, parse_header, save_file
from lunaflux_b200.models.spec import SpecError, LlamaSpec, llama3_8b, mixtral_8x7b, tiny_llama
from lunaflux_b200.utils.json_strict import StrictJsonError, loads_strict


def test_lifecycle_table():
    S = RequestState
    assert can_transition(S.WAITING, S.PREFILL)
    assert can_transition(S.PREFILL, S.PREFILL)
    assert can_transition(S.DECODE, S.FINISHING)
    assert not can_transition(S.WAITING, S.DECODE)
    for t in (S.CANCELLED, S.FINISHED, S.FAILED):
        assert all(not can_transition(t, n) for n in S)


def test_request_validation_categories():
    lim = default_limits(1000, 4096)
    ok = GenerateRequest(1, input_tokens=(1, 2, 3), max_new_tokens=4).validate(lim)
    assert ok.max_new_tokens == 4
    cases = [
        (GenerateRequest(1, input_tokens=(), max_new_tokens=4), ContractField.INPUT_TOKEN, ContractIssue.EMPTY),
        (GenerateRequest(1, input_tokens=(5000,), max_new_tokens=4), ContractField.INPUT_TOKEN,
         ContractIssue.OUT_OF_RANGE),
        (GenerateRequest(1, input_tokens=(1,), max_new_tokens=0), ContractField.MAXIMUM_NEW_TOKENS,
         ContractIssue.OUT_OF_RANGE),
        (GenerateRequest(1, input_tokens=(1,), sampling=SamplingParameters.sample(0.0)), ContractField.TEMPERATURE,
         ContractIssue.OUT_OF_RANGE),
        (GenerateRequest(1, input_tokens=(1,), sampling=SamplingParameters.sample(1.0, top_p=1.5)),
         ContractField.TOP_P, ContractIssue.OUT_OF_RANGE),
        (GenerateRequest(1, input_tokens=(1,), sampling=SamplingParameters(seed=0)), ContractField.SAMPLING_SEED,
         ContractIssue.OUT_OF_RANGE),
        (GenerateRequest(1, input_tokens=(1,), stop=StopConditions(token_ids=(3, 3))), ContractField.STOP_TOKEN,
         ContractIssue.DUPLICATE),
        (GenerateRequest(1, input_text=b"\xff"), ContractField.INPUT_TEXT, ContractIssue.INVALID_FORMAT),
    ]
    for req, field, issue in cases:
        with pytest.raises(ContractError) as e:
            req.validate(lim)
        assert (e.value.field, e.value.issue) == (field, issue)
        assert "\xff" not in str(e.value)  # payload-free errors


def test_derive_seed_nonzero_and_stable():
    seeds = [derive_seed(0, i) for i in range(1000)]
    assert all(s != 0 for s in seeds) and len(set(seeds)) == 1000
    assert derive_seed(0, 5) == derive_seed(0, 5)


def test_strict_json():
    assert loads_strict('{"a": 1}') == {"a": 1}
    with pytest.raises(StrictJsonError):
        loads_strict('{"a": 1, "a": 2}')
    with pytest.raises(StrictJsonError):
        loads_strict('{"a": 1, "\\u0061": 2}')  # escape-equivalent duplicate
    with pytest.raises(StrictJsonError):
        loads_strict('{"a": NaN}')
    with pytest.raises(StrictJsonError):
        loads_strict("[" * 100 + "]" * 100)


def test_config_document():
    doc = {"schema_version": 1, "model": {"preset": "llama3-8b"}, "scheduler": {"max_active_requests": 64},
           "parallel": {"tp": 8}}
    cfg = parse_document(json.dumps(doc))
    assert cfg.parallel.tp == 8 and cfg.scheduler.max_active_requests == 64
    for bad in [dict(doc, extra=1), dict(doc, schema_version=2), {"schema_version": 1},
                dict(doc, scheduler={"bogus": 1}), dict(doc, parallel={"tp": 3})]:
        with pytest.raises(ConfigError):
            parse_document(json.dumps(bad))
    with pytest.raises(ConfigError):
        parse_document('{"schema_version": 1, "model": {"preset": "x"}, "model": {"preset": "y"}}')
    plan = resolve(cfg, kv_bytes_per_page=2 << 20, free_bytes=10 << 30, max_context=2048)
    assert plan.total_pages == 5120 and plan.pages_per_request == 128 and plan.max_rows == 64


def test_safetensors_roundtrip_and_hostile(tmp_path):
    t = {"a": torch.randn(3, 4), "b": torch.randn(5).bfloat16(), "c": torch.arange(6, dtype=torch.int32)}
    p = str(tmp_path / "x.safetensors")
    save_file(t, p, {"format": "pt"})
    with SafetensorsFile(p) as f:
        assert f.metadata == {"format": "pt"}
        for k, v in t.items():
            assert torch.equal(f.tensor(k), v)
    raw = open(p, "rb").read()
    hlen = struct.unpack("<Q", raw[:8])[0]
    with pytest.raises(SafetensorsError):
        parse_header(struct.pack("<Q", 10 ** 12) + raw[8:], len(raw))
    hdr = json.loads(raw[8:8 + hlen])
    hdr["b"]["data_offsets"] = hdr["a"]["data_offsets"][:1] + [hdr["a"]["data_offsets"][0] + 10]
    bad = json.dumps(hdr).encode()
    with pytest.raises(SafetensorsError):
        parse_header(struct.pack("<Q", len(bad)) + bad, 8 + len(bad) + 1000)
    dup = b'{"a":{"dtype":"F32","shape":[1],"data_offsets":[0,4]},"a":{"dtype":"F32","shape":[1],"data_offsets":[0,4]}}'
    with pytest.raises(SafetensorsError):
        parse_header(struct.pack("<Q", len(dup)) + dup, 8 + len(dup) + 4)


def test_specs_and_digests():
    s = llama3_8b()
    assert abs(s.param_count() / 1e9 - 8.03) < 0.05
    assert s.kv_bytes_per_token() == 32 * 2 * 8 * 128 * 2
    assert s.plan_digest() == llama3_8b().plan_digest()
    assert s.plan_digest() != s.with_layers(31).plan_digest()
    assert s.paged_plan_digest(16, 2) != s.paged_plan_digest(16, 1)
    m = mixtral_8x7b()
    assert m.is_moe and abs(m.param_count() / 1e9 - 46.7) < 0.2
    with pytest.raises(SpecError):
        LlamaSpec(hidden=64, layers=1, heads=3, kv_heads=2, head_dim=16, ffn=64, vocab=10)
    assert tiny_llama().group == 2


def test_context_ceiling_consistency():
    """The prompt and every requested token must fit under the ceiling
    (reference: contracts/inference/request.mbt:272-281)."""
    lim = default_limits(1000, 4096)
    GenerateRequest(1, input_tokens=(1,) * 6, max_new_tokens=4, context_ceiling=10).validate(lim)
    for toks, new, ceil in (((1,) * 7, 4, 10), ((1,), 11, 10)):
        with pytest.raises(ContractError) as e:
            GenerateRequest(1, input_tokens=toks, max_new_tokens=new, context_ceiling=ceil).validate(lim)
        assert (e.value.field, e.value.issue) == (ContractField.CONTEXT_CEILING, ContractIssue.INCONSISTENT)
    with pytest.raises(ContractError) as e:
        GenerateRequest(1, input_tokens=(1,), max_new_tokens=4, context_ceiling=5000).validate(lim)
    assert e.value.issue is ContractIssue.OUT_OF_RANGE
