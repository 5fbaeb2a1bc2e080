"""Byte-level BPE: merge semantics, special tokens, round trips, subset admission."""
import json

import pytest

from lunaflux_b200.tokenizer.bpe import Tokenizer, TokenizerError, byte_alphabet


def make_json(merges, added=(), **overrides):
    alpha = byte_alphabet()
    vocab = {alpha[b]: b for b in range(256)}
    nxt = 256
    for a, b in merges:
        if a + b not in vocab:
            vocab[a + b] = nxt
            nxt += 1
    d = {
        "version": "1.0", "truncation": None, "padding": None,
        "added_tokens": [{"id": i, "content": s, "special": True, "single_word": False, "lstrip": False,
                          "rstrip": False, "normalized": False} for s, i in added],
        "normalizer": None,
        "pre_tokenizer": {"type": "ByteLevel", "add_prefix_space": False, "trim_offsets": True, "use_regex": False},
        "post_processor": None,
        "decoder": {"type": "ByteLevel", "add_prefix_space": False, "trim_offsets": True, "use_regex": False},
        "model": {"type": "BPE", "dropout": None, "unk_token": None, "continuing_subword_prefix": None,
                  "end_of_word_suffix": None, "fuse_unk": False, "byte_fallback": False, "ignore_merges": False,
                  "vocab": vocab, "merges": [f"{a} {b}" for a, b in merges]},
    }
    d.update(overrides)
    return json.dumps(d), vocab


MERGES = [("r", "e"), ("a", "t"), ("e", "d"), ("u", "n"), ("at", "ed"), ("re", "l"), ("rel", "ated"),
          ("un", "related")]


def test_ranked_merges_and_spaces():
    text, vocab = make_json(MERGES)
    tok = Tokenizer.from_json(text)
    assert tok.encode("unrelated") == [vocab["unrelated"]]
    ids = tok.encode("unrelated unrelated")
    space = vocab[byte_alphabet()[32]]
    assert ids == [vocab["unrelated"], space, vocab["unrelated"]]
    assert tok.decode(ids) == "unrelated unrelated"


def test_merge_all_occurrences_left_to_right():
    # "aaa" with merge (a, a): non-overlapping left-to-right gives [aa, a]
    text, vocab = make_json([("a", "a")])
    tok = Tokenizer.from_json(text)
    assert tok.encode("aaa") == [vocab["aa"], vocab["a"]]
    assert tok.encode("aaaa") == [vocab["aa"], vocab["aa"]]


def test_unicode_and_zero_byte_roundtrip():
    text, _ = make_json(MERGES)
    tok = Tokenizer.from_json(text)
    for s in ["hé🙂", "line\n\x00end", "A Nuskhuri იესუ", ""]:
        ids = tok.encode(s)
        assert len(ids) == len(s.encode()) or "un" in s
        assert tok.decode(ids) == s


def test_special_tokens_longest_match():
    _, vocab = make_json(MERGES)
    s, sx = len(vocab), len(vocab) + 1          # added ids continue the dense range
    text, vocab = make_json(MERGES, added=[("<s>", s), ("<s>x", sx)])
    tok = Tokenizer.from_json(text)
    assert tok.encode("<s>xunrelated") == [sx, vocab["unrelated"]]
    assert tok.encode("a<s>b") == [vocab["a"], s, vocab["b"]]
    with pytest.raises(TokenizerError):
        tok.encode("a<s>b", allow_special=False)
    assert tok.decode([s]) == "<s>"


def test_token_ids_must_be_dense_from_zero():
    """Reference: tokenizer 'token IDs must be dense within the vocabulary
    range'; an id gap or a negative id is refused at load."""
    _, vocab = make_json(MERGES)
    for added in ([("<s>", len(vocab) + 5)], [("<s>", -1)]):
        text, _ = make_json(MERGES, added=added)
        with pytest.raises(TokenizerError, match="dense"):
            Tokenizer.from_json(text)


@pytest.mark.parametrize("override", [
    {"normalizer": {"type": "NFC"}},
    {"pre_tokenizer": {"type": "ByteLevel", "add_prefix_space": True, "use_regex": False}},
    {"pre_tokenizer": {"type": "Sequence", "pretokenizers": [
        {"type": "Split", "pattern": {"Regex": " "}, "behavior": "Removed", "invert": False},
        {"type": "ByteLevel", "add_prefix_space": False, "use_regex": False}]}},
    {"post_processor": {"type": "TemplateProcessing", "single": [{"Sequence": {"id": "A", "type_id": 0}},
                                                                 {"SpecialToken": {"id": "</s>", "type_id": 0}}]}},
    {"post_processor": {"type": "BertProcessing"}},
    {"pre_tokenizer": {"type": "Whitespace"}},
])
def test_unsupported_subset_rejected(override):
    text, _ = make_json(MERGES, **override)
    with pytest.raises(TokenizerError):
        Tokenizer.from_json(text)


def test_bpe_model_flags_rejected():
    text, _ = make_json(MERGES)
    d = json.loads(text)
    d["model"]["byte_fallback"] = True
    with pytest.raises(TokenizerError):
        Tokenizer.from_json(json.dumps(d))
    d = json.loads(text)
    d["model"]["merges"].append("zz qq")
    with pytest.raises(TokenizerError):
        Tokenizer.from_json(json.dumps(d))
