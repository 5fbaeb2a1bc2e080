"""Byte-level BPE tokenizer over a strict ``tokenizer.json`` subset.

Reference: tokenizer/spec.mbt:66 (TokenizerSpec::new), encode.mbt:28-47,
decode.mbt:3-106, README.mbt.md.  Accepted subset (anything else is rejected
at load): null normalizer and post-processor; ByteLevel pre-tokenizer and
decoder without regex splitting and without prefix space; BPE model without
dropout, unknown token, subword prefix/suffix, byte fallback or
ignore_merges.  Merge semantics are the canonical ones: pick the best-ranked
adjacent pair over the whole symbol list, merge every non-overlapping
occurrence left to right, repeat.  Added (special) tokens are matched
longest-first, lowest id on ties, before BPE runs on the text between them.

The byte <-> symbol alphabet is GPT-2's reversible byte-level map: printable
Latin-1 bytes stand for themselves, the other 68 bytes are shifted to code
points 256 and up.

Beyond the reference's subset, the layout of the Llama 3 and GPT-2 style
tokenizers is accepted too: a pre-tokenizer that splits the text with a
regular expression before the byte-level map (``Split`` with a ``Regex``
pattern and ``Isolated`` behaviour followed by ``ByteLevel`` without regex,
or ``ByteLevel`` with ``use_regex`` and GPT-2's pattern); BPE with
``ignore_merges`` (a pre-token that is itself in the vocabulary is emitted
whole); a ``ByteLevel`` / ``TemplateProcessing`` post-processor whose single
template is an optional leading special token and the sequence (the BOS that
``encode(..., add_special_tokens=True)`` prepends).  Merge results per
pre-token are cached.
"""
from __future__ import annotations

import hashlib
import re
from dataclasses import dataclass
from typing import Dict, Iterable, List, Optional, Sequence, Tuple

from ..utils.json_strict import loads_strict

# GPT-2's pre-tokenisation pattern (ByteLevel with use_regex); it needs the
# `regex` module's Unicode property classes.
GPT2_SPLIT = r"""'s|'t|'re|'ve|'m|'ll|'d| ?\p{L}+| ?\p{N}+| ?[^\s\p{L}\p{N}]+|\s+(?!\S)|\s+"""
_CACHE_MAX = 1 << 16


class TokenizerError(ValueError):
    """A tokenizer failure.  ``kind`` names the failure class (the reference's
    typed errors, tokenizer/types.mbt: ``input_too_long``, ``output_too_long``,
    ``special_token_rejected``, ``unknown_token_id``, ``decoded_too_long``,
    ``invalid_utf8``, ``limit`` ...; ``invalid`` for a malformed document) and
    ``fields`` its integers (``actual`` / ``maximum`` / ``token_id``); neither
    carries text from the input."""

    def __init__(self, message: str, kind: str = "invalid", **fields: int):
        super().__init__(message)
        self.kind = kind
        self.fields = fields


@dataclass(frozen=True)
class TokenizerLimits:
    """Resource bounds checked at load and on every bounded call (reference:
    ``TokenizerLimits``, tokenizer/types.mbt).  The defaults admit the Llama 3
    tokenizer (128256 ids, 280147 merges, 256 special tokens)."""
    max_input_bytes: int = 1 << 26
    max_output_tokens: int = 1 << 24
    max_decoded_bytes: int = 1 << 26
    max_vocab_entries: int = 1 << 21
    max_merge_rules: int = 1 << 21
    max_token_bytes: int = 1 << 12
    max_special_tokens: int = 1 << 16

    def __post_init__(self):
        for k, v in self.__dict__.items():
            if type(v) is not int or v <= 0:
                raise TokenizerError(f"tokenizer limit {k} must be a positive int", "limit")


@dataclass(frozen=True)
class EncodeResult:
    """One bounded encode: the ids, the input's byte length and whether the
    ids were cut at the output limit."""
    token_ids: List[int]
    input_bytes: int
    truncated: bool


#: encode-side special-token policies: emit them, refuse the input, or treat
#: their text as ordinary bytes (no special matching at all)
SPECIAL_POLICIES = ("allow", "reject", "ordinary")
#: decode-side policies: keep the special tokens' text, or drop it
DECODE_SPECIAL_POLICIES = ("preserve", "skip")
TRUNCATION_POLICIES = ("reject", "truncate")


def byte_alphabet() -> Dict[int, str]:
    keep = list(range(ord("!"), ord("~") + 1)) + list(range(0xA1, 0xAC + 1)) + list(range(0xAE, 0xFF + 1))
    table = {}
    shift = 0
    for b in range(256):
        if b in keep:
            table[b] = chr(b)
        else:
            table[b] = chr(256 + shift)
            shift += 1
    return table


_B2U = byte_alphabet()
_U2B = {u: b for b, u in _B2U.items()}


def _piece_bytes(sym: str) -> Optional[bytes]:
    """The bytes a byte-level vocabulary string stands for (None: not one)."""
    try:
        return bytes(_U2B[c] for c in sym)
    except KeyError:
        return None


class Tokenizer:
    def __init__(self, vocab: Dict[str, int], merges: Sequence[Tuple[str, str]], added: Sequence[Tuple[str, int]] = (),
                 digest: str = "", split_pattern: Optional[str] = None, ignore_merges: bool = False,
                 bos_id: Optional[int] = None, limits: Optional[TokenizerLimits] = None):
        self.limits = lim = limits if limits is not None else TokenizerLimits()
        if len(vocab) > lim.max_vocab_entries:
            raise TokenizerError("vocabulary too large", "limit", actual=len(vocab), maximum=lim.max_vocab_entries)
        if len(merges) > lim.max_merge_rules:
            raise TokenizerError("merge table too large", "limit", actual=len(merges), maximum=lim.max_merge_rules)
        if len(added) > lim.max_special_tokens:
            raise TokenizerError("too many special tokens", "limit", actual=len(added),
                                 maximum=lim.max_special_tokens)
        self.vocab = dict(vocab)
        self.split_pattern = split_pattern
        self._split = None
        if split_pattern is not None:
            import regex
            try:
                self._split = regex.compile(split_pattern)
            except regex.error as e:
                raise TokenizerError(f"pre-tokenizer pattern does not compile: {e}") from None
        self.ignore_merges = bool(ignore_merges)
        self.bos_id = bos_id
        self._cache: Dict[bytes, List[int]] = {}
        self.id_to_token: Dict[int, str] = {}
        for t, i in self.vocab.items():
            if i in self.id_to_token:
                raise TokenizerError("duplicate token id")
            self.id_to_token[i] = t
        for b, u in _B2U.items():
            if u not in self.vocab:
                raise TokenizerError("vocabulary lacks the byte-level alphabet", "missing_byte", byte_value=b)
        for t, i in self.vocab.items():
            if not t:
                raise TokenizerError("empty token piece", "empty_piece", token_id=i)
            if len(t) > lim.max_token_bytes:   # symbols: one per byte of the piece
                raise TokenizerError("token piece too long", "limit", token_id=i, actual=len(t),
                                     maximum=lim.max_token_bytes)
        self.ranks: Dict[Tuple[str, str], int] = {}
        for r, (a, b) in enumerate(merges):
            if a not in self.vocab or b not in self.vocab or (a + b) not in self.vocab:
                raise TokenizerError("merge refers to a token outside the vocabulary")
            if (a, b) in self.ranks:
                raise TokenizerError("duplicate merge")
            self.ranks[(a, b)] = r
        self.added = sorted(((s, i) for s, i in added), key=lambda x: (-len(x[0].encode()), x[1]))
        self.added_ids = {i for _, i in added}
        self._special_ids = {t.encode(): i for t, i in self.added}
        self._special_re = re.compile(b"|".join(re.escape(t.encode()) for t, _ in self.added)) if self.added else None
        seen_special: Dict[str, int] = {}
        for s, i in added:
            if not s:
                raise TokenizerError("empty special token", "empty_piece", token_id=i)
            if len(s.encode()) > lim.max_token_bytes:
                raise TokenizerError("special token too long", "limit", token_id=i, actual=len(s.encode()),
                                     maximum=lim.max_token_bytes)
            if seen_special.setdefault(s, i) != i:
                raise TokenizerError("two special tokens with the same text", "duplicate_piece",
                                     first=seen_special[s], duplicate=i)
            prev = self.id_to_token.get(i)
            if prev is not None and prev != s and _piece_bytes(prev) != s.encode():
                # an id already taken by another piece (a vocabulary entry with
                # different bytes, or an earlier special token)
                raise TokenizerError("duplicate token id", "duplicate_id", token_id=i)
            self.id_to_token.setdefault(i, s)
        # ids are dense from 0 (every id below the largest decodes to a token)
        ids = self.id_to_token.keys()
        if any(type(i) is not int or i < 0 for i in ids) or (ids and max(ids) + 1 != len(ids)):
            raise TokenizerError("token ids must be dense from 0")
        self.digest = digest
        # The merge loop runs in the C++ host core when it is built (same
        # semantics, on ids); the Python loop below is its reference.
        self._byte_ids = [self.vocab[_B2U[b]] for b in range(256)]
        self._native = None
        try:
            from .. import _host
            self._native = _host.BpeEncoder([(self.vocab[a], self.vocab[b], self.vocab[a + b])
                                             for (a, b) in sorted(self.ranks, key=self.ranks.get)])
        except ImportError:
            pass
        self.vocab_size = max(self.id_to_token) + 1 if self.id_to_token else 0
        if bos_id is not None and bos_id not in self.id_to_token:
            raise TokenizerError("the post-processor's special token is not in the vocabulary")

    # ------------------------------------------------------------------ loading
    @classmethod
    def from_json(cls, text: str | bytes) -> "Tokenizer":
        raw = text.encode() if isinstance(text, str) else bytes(text)
        d = loads_strict(raw)
        if d.get("normalizer") is not None:
            raise TokenizerError("normalizer must be null")
        split = _pre_tokenizer(d.get("pre_tokenizer"))
        dec = d.get("decoder")
        if not isinstance(dec, dict) or dec.get("type") != "ByteLevel":
            raise TokenizerError("decoder must be ByteLevel")
        m = d.get("model")
        if not isinstance(m, dict) or m.get("type") != "BPE":
            raise TokenizerError("model must be BPE")
        for k in ("dropout", "unk_token", "continuing_subword_prefix", "end_of_word_suffix"):
            if m.get(k) is not None:
                raise TokenizerError(f"BPE {k} is not supported")
        for k in ("fuse_unk", "byte_fallback"):
            if m.get(k, False):
                raise TokenizerError(f"BPE {k} is not supported")
        merges = []
        for mm in m.get("merges", []):
            if isinstance(mm, str):
                parts = mm.split(" ")
                if len(parts) != 2:
                    raise TokenizerError("malformed merge")
                merges.append((parts[0], parts[1]))
            elif isinstance(mm, list) and len(mm) == 2:
                merges.append((mm[0], mm[1]))
            else:
                raise TokenizerError("malformed merge")
        added = []
        for a in d.get("added_tokens", []) or []:
            if a.get("normalized") or a.get("lstrip") or a.get("rstrip") or a.get("single_word"):
                raise TokenizerError("added-token flags are not supported")
            added.append((a["content"], int(a["id"])))
        bos = _post_processor(d.get("post_processor"))
        return cls(m["vocab"], merges, added, hashlib.sha256(raw).hexdigest(), split_pattern=split,
                   ignore_merges=bool(m.get("ignore_merges", False)), bos_id=bos)

    @classmethod
    def from_file(cls, path: str) -> "Tokenizer":
        with open(path, "rb") as f:
            return cls.from_json(f.read())

    # ------------------------------------------------------------------ encode
    def _bpe(self, data: bytes) -> List[int]:
        if self._native is not None:
            return self._native.encode([self._byte_ids[b] for b in data])
        return self._bpe_reference(data)

    def _bpe_reference(self, data: bytes) -> List[int]:
        syms = [_B2U[b] for b in data]
        if len(syms) > 1:
            ranks = self.ranks
            while True:
                best = None
                for a, b in zip(syms, syms[1:]):
                    r = ranks.get((a, b))
                    if r is not None and (best is None or r < best[0]):
                        best = (r, a, b)
                if best is None:
                    break
                _, a, b = best
                out = []
                i = 0
                n = len(syms)
                while i < n:
                    if i + 1 < n and syms[i] == a and syms[i + 1] == b:
                        out.append(a + b)
                        i += 2
                    else:
                        out.append(syms[i])
                        i += 1
                syms = out
        return [self.vocab[s] for s in syms]

    def _word(self, data: bytes) -> List[int]:
        """One pre-token (cached)."""
        ids = self._cache.get(data)
        if ids is None:
            whole = self.vocab.get("".join(_B2U[b] for b in data)) if self.ignore_merges else None
            ids = [whole] if whole is not None else self._bpe(data)
            if len(self._cache) >= _CACHE_MAX:
                self._cache.clear()
            self._cache[data] = ids
        return ids

    def _segment(self, data: bytes) -> List[int]:
        """Text between special tokens: pre-tokenise, then BPE per piece."""
        if self._split is None:
            return self._word(data) if self.ignore_merges else self._bpe(data)
        # bytes that are not UTF-8 travel through the split as lone surrogates
        text = data.decode("utf-8", errors="surrogateescape")
        ids: List[int] = []
        for piece in self._split.findall(text):
            if piece:
                ids += self._word(piece.encode("utf-8", errors="surrogateescape"))
        return ids

    def encode_bytes(self, data: bytes, allow_special: bool = True, add_special_tokens: bool = False) -> List[int]:
        ids = self._encode_bytes(data, allow_special)
        if add_special_tokens and self.bos_id is not None:
            ids.insert(0, self.bos_id)
        return ids

    def _encode_bytes(self, data: bytes, allow_special: bool) -> List[int]:
        if not self.added:
            return self._segment(data)
        ids: List[int] = []
        start = 0
        # one scan for the leftmost special token; the alternation lists the
        # longest first, so the first alternative that matches is the longest
        for m in self._special_re.finditer(data):
            tid = self._special_ids[m.group()]
            if not allow_special:
                raise TokenizerError("input contains a special token", "special_token_rejected", token_id=tid)
            if start < m.start():
                ids += self._segment(data[start:m.start()])
            ids.append(tid)
            start = m.end()
        if start < len(data):
            ids += self._segment(data[start:])
        return ids

    def encode(self, text: str, allow_special: bool = True, add_special_tokens: bool = False) -> List[int]:
        """Token ids of ``text``; ``add_special_tokens`` applies the
        post-processor's template (a leading BOS when it has one)."""
        return self.encode_bytes(text.encode("utf-8"), allow_special, add_special_tokens)

    def encode_bounded(self, data: bytes | str, special_policy: str = "allow", output_limit: Optional[int] = None,
                       truncation: str = "reject", add_special_tokens: bool = False) -> EncodeResult:
        """Bounded encode (reference: ``TokenizerSpec::encode_bytes`` /
        ``encode_text``, tokenizer/encode.mbt).  ``special_policy``: "allow"
        emits special tokens (longest match), "reject" fails at the first one
        with its id, "ordinary" encodes their text as plain bytes.  The input
        must fit ``max_input_bytes``; ``output_limit`` (default and ceiling:
        ``max_output_tokens``) bounds the ids: "reject" fails with the full
        count, "truncate" keeps the first ``output_limit`` and sets
        ``truncated``."""
        if isinstance(data, str):
            data = data.encode("utf-8")
        data = bytes(data)
        lim = self.limits
        if special_policy not in SPECIAL_POLICIES:
            raise TokenizerError(f"special_policy must be one of {SPECIAL_POLICIES}", "invalid_argument")
        if truncation not in TRUNCATION_POLICIES:
            raise TokenizerError(f"truncation must be one of {TRUNCATION_POLICIES}", "invalid_argument")
        if output_limit is None:
            output_limit = lim.max_output_tokens
        if type(output_limit) is not int or output_limit <= 0 or output_limit > lim.max_output_tokens:
            raise TokenizerError("output limit outside 1..max_output_tokens", "invalid_output_limit",
                                 requested=output_limit if type(output_limit) is int else -1,
                                 maximum=lim.max_output_tokens)
        if len(data) > lim.max_input_bytes:
            raise TokenizerError("input too long", "input_too_long", actual=len(data), maximum=lim.max_input_bytes)
        if special_policy == "ordinary":
            ids = self._segment(data) if data else []
        else:
            ids = self._encode_bytes(data, special_policy == "allow")
        if add_special_tokens and self.bos_id is not None:
            ids.insert(0, self.bos_id)
        if len(ids) > output_limit:
            if truncation == "reject":
                raise TokenizerError("output too long", "output_too_long", actual=len(ids), maximum=output_limit)
            return EncodeResult(ids[:output_limit], len(data), True)
        return EncodeResult(ids, len(data), False)

    # ------------------------------------------------------------------ decode
    def token_bytes(self, tid: int) -> bytes:
        t = self.id_to_token.get(tid) if type(tid) is int else None
        if t is None:
            raise TokenizerError("unknown token id", "unknown_token_id", token_id=tid if type(tid) is int else -1)
        if tid in self.added_ids:
            return t.encode("utf-8")
        try:
            return bytes(_U2B[c] for c in t)
        except KeyError:
            raise TokenizerError("token outside the byte-level alphabet") from None

    def decode_bytes(self, ids: Iterable[int], special_policy: str = "preserve") -> bytes:
        """The bytes of ``ids`` (reference: tokenizer/decode.mbt): every id is
        checked first, "skip" drops special tokens, and the output is bounded
        by ``max_decoded_bytes`` (nothing is returned past the bound)."""
        if special_policy not in DECODE_SPECIAL_POLICIES:
            raise TokenizerError(f"special_policy must be one of {DECODE_SPECIAL_POLICIES}", "invalid_argument")
        skip = special_policy == "skip"
        cap = self.limits.max_decoded_bytes
        out = []
        n = 0
        for i in ids:
            piece = self.token_bytes(i)
            if skip and i in self.added_ids:
                continue
            n += len(piece)
            if n > cap:
                raise TokenizerError("decoded output too long", "decoded_too_long", maximum=cap)
            out.append(piece)
        return b"".join(out)

    def decode_text(self, ids: Iterable[int], special_policy: str = "preserve") -> str:
        """Strict text decode: the bytes must be valid UTF-8 (a token sequence
        that ends inside a character, or carries arbitrary bytes, fails)."""
        data = self.decode_bytes(ids, special_policy)
        try:
            return data.decode("utf-8")
        except UnicodeDecodeError:
            raise TokenizerError("decoded bytes are not valid UTF-8", "invalid_utf8") from None

    def decoded_piece_bytes(self, tid: int, special_policy: str = "preserve") -> int:
        """Byte length of one token's decoded piece (0 for a skipped special)."""
        return len(self.decode_bytes([tid], special_policy))

    def decode(self, ids: Iterable[int]) -> str:
        """Lenient text decode: invalid UTF-8 becomes U+FFFD."""
        return self.decode_bytes(ids).decode("utf-8", errors="replace")


def _pre_tokenizer(p) -> Optional[str]:
    """The split pattern of an accepted pre-tokenizer (None: no split)."""
    def byte_level(q, allow_regex):
        if not isinstance(q, dict) or q.get("type") != "ByteLevel" or q.get("add_prefix_space", False):
            return False
        return allow_regex or not q.get("use_regex", True)

    if isinstance(p, dict) and p.get("type") == "ByteLevel":
        if not byte_level(p, True):
            raise TokenizerError("pre_tokenizer: ByteLevel with a prefix space is not supported")
        return GPT2_SPLIT if p.get("use_regex", True) else None
    if isinstance(p, dict) and p.get("type") == "Sequence":
        seq = p.get("pretokenizers")
        if isinstance(seq, list) and len(seq) == 2 and byte_level(seq[1], False):
            sp = seq[0]
            pat = sp.get("pattern") if isinstance(sp, dict) else None
            if isinstance(sp, dict) and sp.get("type") == "Split" and isinstance(pat, dict) and \
                    isinstance(pat.get("Regex"), str) and sp.get("behavior") == "Isolated" and not sp.get("invert"):
                return pat["Regex"]
    raise TokenizerError("pre_tokenizer must be ByteLevel, or a regex Split (Isolated) then ByteLevel without regex")


def _post_processor(p) -> Optional[int]:
    """The BOS id of an accepted post-processor (None: nothing is added)."""
    if p is None:
        return None
    if not isinstance(p, dict):
        raise TokenizerError("post_processor must be an object or null")
    kind = p.get("type")
    if kind == "ByteLevel":
        return None
    if kind == "Sequence":
        bos = None
        for q in p.get("processors") or []:
            b = _post_processor(q)
            if b is not None:
                if bos is not None:
                    raise TokenizerError("post_processor: more than one template")
                bos = b
        return bos
    if kind == "TemplateProcessing":
        single = p.get("single")
        if not isinstance(single, list) or not single or single[-1] != {"Sequence": {"id": "A", "type_id": 0}}:
            raise TokenizerError("post_processor: the single template must end with the sequence")
        if len(single) == 1:
            return None
        head = single[0].get("SpecialToken") if isinstance(single[0], dict) else None
        if len(single) != 2 or not isinstance(head, dict):
            raise TokenizerError("post_processor: only a leading special token is supported")
        spec = (p.get("special_tokens") or {}).get(head.get("id"))
        ids = spec.get("ids") if isinstance(spec, dict) else None
        if not isinstance(ids, list) or len(ids) != 1 or type(ids[0]) is not int:
            raise TokenizerError("post_processor: the special token needs exactly one id")
        return ids[0]
    raise TokenizerError(f"post_processor {kind!r} is not supported")


def synthetic_byte_tokenizer(vocab_size: int = 256) -> Tokenizer:
    """A tokenizer whose ids 0..255 are the raw bytes (used with random-init
    models whose vocabulary has no text meaning)."""
    vocab = {_B2U[b]: b for b in range(256)}
    t = Tokenizer(vocab, [], digest=hashlib.sha256(b"lunaflux-byte-tokenizer").hexdigest())
    return t
