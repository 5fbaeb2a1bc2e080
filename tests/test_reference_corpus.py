"""Pinned upstream corpora: numbers produced outside this repository.

``tests/fixtures/tiny_random_llama2`` holds the exact upstream bytes of
``stas/tiny-random-llama-2`` (Apache-2.0; config.json and the 210,712-byte
BF16 model.safetensors at revision 3579d71f) with golden values that
``transformers`` 4.53.2 on CPU torch 2.7.1 computed from them: last-position
logits at eleven vocabulary indices, the argmax and a four-token greedy
continuation for three prompts, compared at abs / rel 1e-5.  The reference
checks the same corpus in tests/reference_corpus/reference_corpus_test.mbt
and reference_text_pipeline_test.mbt (expected values:
tests/reference_corpus/corpus.json, provenance MANIFEST.md:1-85).

``tests/fixtures/bytelevel_bpe`` is the compact ByteLevel-BPE tokenizer
derived from Hugging Face ``tokenizers`` 0.22.2 with encodings that library
produced (reference: tests/reference_tokenizer/corpus.json, MANIFEST.md:1-45).

Every fixture is checked against its pinned SHA-256 before use, so a changed
file cannot silently move the goal posts.
"""
import hashlib
import json
import os
import shutil

import pytest
import torch

FIX = os.path.join(os.path.dirname(os.path.abspath(__file__)), "fixtures")
LLAMA = os.path.join(FIX, "tiny_random_llama2")
BPE = os.path.join(FIX, "bytelevel_bpe")

SHA256 = {
    os.path.join(LLAMA, "config.json"): "9197475bfcc987a4f9361dbc22b33397b101372c137c228b6a6fd7e4adf21622",
    os.path.join(LLAMA, "model.safetensors"): "852db1b39acb2336abc997440c6f6d6e4ab640f91e5e2aa9e2488d5794159d30",
    os.path.join(LLAMA, "corpus.json"): "f4ade303b1b7b3264e86caa15b77cdb2805244e1142b9b74225ed3f36438f1d0",
    os.path.join(LLAMA, "tokenizer_semantics_probe.json"):
        "4ac8db0bb211b5bd064b58eaab43a3bd38de593593eceadc7364848fcf4f954f",
    os.path.join(LLAMA, "compatible_bytelevel_tokenizer.json"):
        "82000898a396651e5d3b149c5dec02998427406c78ccdf14084cbf85c63d2686",
    os.path.join(BPE, "tokenizer.json"): "72e19c379865733c37776d8386a87707ac50703aed1633fabb5c708b1479e142",
    os.path.join(BPE, "corpus.json"): "c18cec0a5b3d2bbcab51d80153929f4ec6c81af91e5725a83508d07dfb67fbd9",
}


def _read(path):
    with open(path, "rb") as f:
        data = f.read()
    assert hashlib.sha256(data).hexdigest() == SHA256[path], f"{path} differs from its pinned bytes"
    return data


@pytest.fixture(scope="module")
def corpus():
    return json.loads(_read(os.path.join(LLAMA, "corpus.json")))


@pytest.fixture(scope="module")
def checkpoint(tmp_path_factory):
    """The upstream model directory as a user would hand it over: config,
    weights and (here) the byte-level tokenizer that this runtime admits."""
    from lunaflux_b200.models.checkpoint import CheckpointDir
    d = tmp_path_factory.mktemp("tiny_random_llama2")
    for name in ("config.json", "model.safetensors"):
        _read(os.path.join(LLAMA, name))
        shutil.copyfile(os.path.join(LLAMA, name), d / name)
    _read(os.path.join(LLAMA, "compatible_bytelevel_tokenizer.json"))
    shutil.copyfile(os.path.join(LLAMA, "compatible_bytelevel_tokenizer.json"), d / "tokenizer.json")
    ck = CheckpointDir(str(d))
    yield ck
    ck.close()


def test_fixture_digests():
    for path in SHA256:
        _read(path)


def test_checkpoint_admission(checkpoint):
    from lunaflux_b200.models.admission import Rejection, admit
    spec = checkpoint.spec(dtype="fp32")
    assert (spec.layers, spec.hidden, spec.heads, spec.kv_heads, spec.vocab) == (2, 16, 4, 4, 3000)
    assert spec.ffn == 64 and not spec.is_moe
    # bf16 on disk, 2 layers x 9 tensors + embedding, final norm, LM head
    assert len(checkpoint.names()) == 21
    assert {checkpoint.tensor(n).dtype for n in checkpoint.names()} == {torch.bfloat16}
    cpu = admit(spec, max_context=256, kernels=False)
    assert cpu.ok, cpu.details
    # the sm_100a kernels want head_dim 128 and a hidden size that tiles by
    # 256: this model runs on the reference operators only, and says so
    gpu = admit(spec, max_context=256)
    assert not gpu.ok and {Rejection.HEAD_DIM, Rejection.GEMM_ALIGN} <= set(gpu.reasons)
    assert checkpoint.content_digest() == SHA256[os.path.join(LLAMA, "model.safetensors")]


def _close(got, want, atol, rtol):
    return abs(got - want) <= atol + rtol * abs(want)


def test_oracle_logits_match_transformers(checkpoint, corpus):
    from lunaflux_b200.oracle.reference import ReferenceModel
    tol = corpus["logit_tolerance"]
    spec = checkpoint.spec(dtype="fp32")
    ref = ReferenceModel(spec, {n: checkpoint.tensor(n) for n in checkpoint.names()})
    for case in corpus["model_cases"]:
        last = ref.forward(case["input_ids"])[-1]
        assert last.shape == (3000,)
        for idx, want in case["sampled_logits"].items():
            got = float(last[int(idx)])
            assert _close(got, want, tol["absolute"], tol["relative"]), (case["input_ids"], idx, got, want)
        assert int(torch.argmax(last)) == case["greedy_token"]
        assert ref.generate_greedy(case["input_ids"], 4) == case["greedy_continuation"]


def _cpu_engine(checkpoint, spec):
    from lunaflux_b200.config import CacheConfig, SchedulerConfig
    from lunaflux_b200.engine.engine import EngineOptions, LLMEngine
    from lunaflux_b200.models.weights import build_runtime
    from lunaflux_b200.ops.torch_ops import TorchOps
    w = build_runtime(spec, checkpoint.source())
    return LLMEngine(w, TorchOps(), "cpu", SchedulerConfig(step_token_budget=16, max_active_requests=4,
                                                          prefill_chunk_tokens=16, emergency_decode_page_reserve=1),
                     CacheConfig(), EngineOptions(max_context=64, num_pages=32, graph_sizes=()))


def test_engine_greedy_matches_transformers(checkpoint, corpus):
    """The paged engine (scheduler, KV pages, chunked prefill, batched decode)
    reaches the transformers continuations for all three prompts at once."""
    spec = checkpoint.spec(dtype="fp32")
    eng = _cpu_engine(checkpoint, spec)
    cases = corpus["model_cases"]
    outs = eng.generate([c["input_ids"] for c in cases], 4)
    assert outs == [c["greedy_continuation"] for c in cases]


def test_text_reaches_transformers_tokens(checkpoint, corpus):
    """Text in, text out: the admitted byte-level tokenizer maps "Luna*c" onto
    the third model case's ids, whose continuation transformers pinned."""
    tok = checkpoint.tokenizer()
    assert tok.vocab_size == 3000
    ids = tok.encode("Luna*c", add_special_tokens=False)
    assert ids == [1, 42, 99]
    case = next(c for c in corpus["model_cases"] if c["input_ids"] == ids)
    eng = _cpu_engine(checkpoint, checkpoint.spec(dtype="fp32"))
    out = eng.generate([ids], 4)[0]
    assert out == case["greedy_continuation"]
    assert tok.decode(out) == "".join(tok.token_bytes(t).decode("utf-8", "replace") for t in out)


def test_upstream_tokenizer_semantics_are_rejected(corpus):
    """The upstream SentencePiece-style tokenizer (prepend / replace
    normaliser, byte fallback, unknown fusion, template BOS) is outside the
    admitted byte-level subset and is refused, not approximated."""
    from lunaflux_b200.tokenizer.bpe import Tokenizer, TokenizerError
    probe = _read(os.path.join(LLAMA, "tokenizer_semantics_probe.json"))
    with pytest.raises(TokenizerError):
        Tokenizer.from_json(probe)
    # each offending feature alone is refused as well
    base = json.loads(probe)
    for mutate in (lambda d: d["model"].update(byte_fallback=True, fuse_unk=False, unk_token=None),
                   lambda d: d["model"].update(fuse_unk=True, byte_fallback=False, unk_token=None),
                   lambda d: d["model"].update(unk_token="<unk>", fuse_unk=False, byte_fallback=False)):
        d = json.loads(probe)
        d["normalizer"] = None
        d["decoder"] = {"type": "ByteLevel", "add_prefix_space": False, "trim_offsets": True, "use_regex": False}
        mutate(d)
        with pytest.raises(TokenizerError):
            Tokenizer.from_json(json.dumps(d))
    assert base["normalizer"] is not None
    # the upstream encodings start with the template BOS (id 1), which the
    # byte-level subset does not insert
    assert all(c["token_ids"][0] == 1 for c in corpus["tokenizer_cases"])


def test_bytelevel_bpe_matches_hf_tokenizers():
    from lunaflux_b200.tokenizer.bpe import Tokenizer
    tok = Tokenizer.from_json(_read(os.path.join(BPE, "tokenizer.json")))
    cases = json.loads(_read(os.path.join(BPE, "corpus.json")))["cases"]
    assert len(cases) == 5
    for c in cases:
        assert c["text"].encode("utf-8").hex() == c["utf8_hex"]
        assert tok.encode(c["text"], add_special_tokens=False) == c["ids"], c["name"]
        assert tok.decode(c["ids"]) == c["decoded"], c["name"]
        # the native merge loop and the Python restatement agree
        data = c["text"].encode("utf-8")
        assert tok._bpe_reference(data) == tok._bpe(data), c["name"]


def test_cli_reference_on_the_pinned_model(corpus):
    """`lunaflux reference ROOT CONFIG TOKENIZER WEIGHTS SHA... N IDS`, with the
    digests pinned above, reaches each model case's transformers continuation."""
    from lunaflux_b200 import cli
    names = ("config.json", "compatible_bytelevel_tokenizer.json", "model.safetensors")
    shas = [SHA256[os.path.join(LLAMA, n)] for n in names]
    for case in corpus["model_cases"]:
        lines = []
        ids = ",".join(map(str, case["input_ids"]))
        gen = cli.reference(LLAMA, *names, *shas, "4", ids, out=lines.append)
        assert gen == case["greedy_continuation"]
        assert lines[-1] == "generated tokens: " + ",".join(map(str, gen))
