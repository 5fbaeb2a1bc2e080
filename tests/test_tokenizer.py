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


# --------------------------------------------------------------------------
# Bounded encode / decode (reference: tokenizer/tokenizer_test.mbt "special
# token policy is explicit and longest-match", "output and input bounds reject
# or truncate deterministically", "decode rejects unknown IDs and decoded byte
# overflow", "Unicode uses exact UTF-8 bytes and arbitrary bytes round trip").

from lunaflux_b200.tokenizer.bpe import EncodeResult, TokenizerLimits  # noqa: E402


def _special_tok(limits=None):
    _, vocab = make_json(MERGES)
    eos, e = len(vocab), len(vocab) + 1
    text, vocab = make_json(MERGES, added=[("<eos>", eos), ("<e", e)])
    tok = Tokenizer.from_json(text)
    if limits is not None:
        tok = Tokenizer(tok.vocab, [tuple(k) for k in sorted(tok.ranks, key=tok.ranks.get)],
                        [("<eos>", eos), ("<e", e)], limits=limits)
    return tok, vocab, eos, e


def test_special_policies_encode():
    tok, vocab, eos, e = _special_tok()
    r = tok.encode_bounded("unrelated<eos><e", special_policy="allow")
    assert r == EncodeResult([vocab["unrelated"], eos, e], 16, False)
    # ordinary: the special text is plain bytes, nothing is matched
    r = tok.encode_bounded("<e>", special_policy="ordinary")
    assert r.token_ids == [vocab["<"], vocab["e"], vocab[">"]]
    # reject: fails at the first special token, naming its id
    with pytest.raises(TokenizerError) as ei:
        tok.encode_bounded("prefix<eos>", special_policy="reject")
    assert ei.value.kind == "special_token_rejected" and ei.value.fields == {"token_id": eos}
    # longest match: "<eos>" wins over its prefix "<e"
    assert tok.encode_bounded("<eos>").token_ids == [eos]
    with pytest.raises(TokenizerError, match="special_policy"):
        tok.encode_bounded("x", special_policy="maybe")


def test_output_bound_truncates_or_rejects():
    tok, vocab, _, _ = _special_tok()
    r = tok.encode_bounded("unrelated!", special_policy="ordinary", output_limit=1, truncation="truncate")
    assert r == EncodeResult([vocab["unrelated"]], 10, True)
    with pytest.raises(TokenizerError) as ei:
        tok.encode_bounded("unrelated!", output_limit=1)
    assert ei.value.kind == "output_too_long" and ei.value.fields == {"actual": 2, "maximum": 1}
    # exactly at the limit is not truncated
    assert tok.encode_bounded("unrelated!", output_limit=2, truncation="truncate").truncated is False
    for bad in (0, -1, tok.limits.max_output_tokens + 1, 1.5):
        with pytest.raises(TokenizerError) as ei:
            tok.encode_bounded("a", output_limit=bad)
        assert ei.value.kind == "invalid_output_limit"


def test_input_bound():
    tok, _, _, _ = _special_tok(TokenizerLimits(max_input_bytes=2))
    assert tok.encode_bounded(b"ab").input_bytes == 2
    with pytest.raises(TokenizerError) as ei:
        tok.encode_bounded(b"abc")
    assert ei.value.kind == "input_too_long" and ei.value.fields == {"actual": 3, "maximum": 2}


def test_decode_special_skip_and_unknown_ids():
    tok, vocab, eos, e = _special_tok()
    ids = tok.encode("unrelated<eos>")
    assert tok.decode_text(ids, special_policy="skip") == "unrelated"
    assert tok.decode_text(ids) == "unrelated<eos>"
    assert tok.decoded_piece_bytes(eos, "skip") == 0
    assert tok.decoded_piece_bytes(vocab["unrelated"]) == 9
    for bad in (9999, -1, tok.vocab_size):
        with pytest.raises(TokenizerError) as ei:
            tok.decode_bytes([vocab["a"], bad])
        assert ei.value.kind == "unknown_token_id" and ei.value.fields == {"token_id": bad}
    # an unknown id fails even where it would be skipped
    with pytest.raises(TokenizerError):
        tok.decode_bytes([9999], special_policy="skip")


def test_decoded_byte_bound():
    tok, vocab, _, _ = _special_tok(TokenizerLimits(max_decoded_bytes=2))
    assert tok.decode_bytes([vocab["a"], vocab["b"]]) == b"ab"
    with pytest.raises(TokenizerError) as ei:
        tok.decode_bytes([vocab["a"], vocab["b"], vocab["c"]])
    assert ei.value.kind == "decoded_too_long" and ei.value.fields == {"maximum": 2}


def test_arbitrary_bytes_round_trip_but_strict_text_fails():
    tok, _, _, _ = _special_tok()
    arbitrary = bytes([0xFF, 0x00, 0xC3, 0x28, 0x80])
    r = tok.encode_bounded(arbitrary, special_policy="ordinary")
    assert len(r.token_ids) == 5 and tok.decode_bytes(r.token_ids) == arbitrary
    with pytest.raises(TokenizerError) as ei:
        tok.decode_text(r.token_ids)
    assert ei.value.kind == "invalid_utf8"
    assert tok.decode(r.token_ids) == arbitrary.decode("utf-8", errors="replace")
    # a character split across tokens decodes strictly only when complete
    ids = tok.encode("é")
    assert len(ids) == 2 and tok.decode_text(ids) == "é"
    with pytest.raises(TokenizerError):
        tok.decode_text(ids[:1])


def test_load_limits_and_duplicates_fail_closed():
    text, vocab = make_json(MERGES)
    base = Tokenizer.from_json(text)
    merges = [tuple(k) for k in sorted(base.ranks, key=base.ranks.get)]
    with pytest.raises(TokenizerError) as ei:
        Tokenizer(vocab, merges, limits=TokenizerLimits(max_vocab_entries=256))
    assert ei.value.kind == "limit" and ei.value.fields["actual"] == len(vocab)
    with pytest.raises(TokenizerError) as ei:
        Tokenizer(vocab, merges, limits=TokenizerLimits(max_merge_rules=len(merges) - 1))
    assert ei.value.kind == "limit"
    with pytest.raises(TokenizerError) as ei:
        Tokenizer(vocab, merges, limits=TokenizerLimits(max_token_bytes=8))   # "unrelated" is 9
    assert ei.value.kind == "limit" and ei.value.fields["actual"] == 9
    with pytest.raises(TokenizerError) as ei:
        Tokenizer(vocab, merges, [("<a>", len(vocab)), ("<b>", len(vocab) + 1)],
                  limits=TokenizerLimits(max_special_tokens=1))
    assert ei.value.kind == "limit"
    # two special tokens with one text, or one id for two pieces
    with pytest.raises(TokenizerError) as ei:
        Tokenizer(vocab, merges, [("<a>", len(vocab)), ("<a>", len(vocab) + 1)])
    assert ei.value.kind == "duplicate_piece"
    with pytest.raises(TokenizerError) as ei:
        Tokenizer(vocab, merges, [("<a>", vocab["a"])])
    assert ei.value.kind == "duplicate_id"
    with pytest.raises(TokenizerError) as ei:
        Tokenizer(vocab, merges, [("", len(vocab))])
    assert ei.value.kind == "empty_piece"
    # a missing byte symbol names the byte
    partial = dict(vocab)
    del partial[byte_alphabet()[255]]
    with pytest.raises(TokenizerError) as ei:
        Tokenizer(partial, [])
    assert ei.value.kind == "missing_byte" and ei.value.fields == {"byte_value": 255}
    for bad in (0, -3, 1.0):
        with pytest.raises(TokenizerError):
            TokenizerLimits(max_input_bytes=bad)


def test_special_token_also_in_vocab_is_admitted():
    """GPT-2 style: the special token is a vocabulary entry with the same id
    and bytes; that is one piece, not a duplicate."""
    text, vocab = make_json(MERGES)
    vocab = dict(vocab)
    eot = len(vocab)
    vocab["<|endoftext|>"] = eot
    tok = Tokenizer(vocab, [], [("<|endoftext|>", eot)])
    assert tok.encode("a<|endoftext|>") == [vocab["a"], eot]
    assert tok.decode_text([eot], special_policy="skip") == ""


def test_special_matching_equals_a_position_scan():
    """The compiled special-token scan picks, at the leftmost position where
    any special token starts, the longest one: the same ids as trying every
    special token at every byte."""
    import random
    _, vocab = make_json(MERGES)
    n = len(vocab)
    specials = [("<a>", n), ("<a>b", n + 1), ("<", n + 2), ("a<a", n + 3), ("é|", n + 4), ("|é|", n + 5)]
    text, vocab = make_json(MERGES, added=specials)
    tok = Tokenizer.from_json(text)
    order = sorted(((s.encode(), i) for s, i in specials), key=lambda x: -len(x[0]))

    def scan(data):
        ids, start, i = [], 0, 0
        while i < len(data):
            hit = next(((s, t) for s, t in order if data.startswith(s, i)), None)
            if hit is None:
                i += 1
                continue
            if start < i:
                ids += tok._segment(data[start:i])
            ids.append(hit[1])
            i += len(hit[0])
            start = i
        return ids + (tok._segment(data[start:]) if start < len(data) else [])

    rng = random.Random(5)
    pieces = ["<", "a", ">", "b", "é", "|", "un", "related", " "]
    for _ in range(500):
        s = "".join(rng.choice(pieces) for _ in range(rng.randint(0, 14))).encode()
        assert tok.encode_bytes(s) == scan(s), s
