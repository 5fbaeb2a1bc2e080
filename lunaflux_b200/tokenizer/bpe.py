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
"""
from __future__ import annotations

import hashlib
from typing import Dict, Iterable, List, Optional, Sequence, Tuple

from ..utils.json_strict import loads_strict


class TokenizerError(ValueError):
    pass


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


class Tokenizer:
    def __init__(self, vocab: Dict[str, int], merges: Sequence[Tuple[str, str]], added: Sequence[Tuple[str, int]] = (),
                 digest: str = ""):
        self.vocab = dict(vocab)
        self.id_to_token: Dict[int, str] = {}
        for t, i in self.vocab.items():
            if i in self.id_to_token:
                raise TokenizerError("duplicate token id")
            self.id_to_token[i] = t
        for b, u in _B2U.items():
            if u not in self.vocab:
                raise TokenizerError("vocabulary lacks the byte-level alphabet")
        self.ranks: Dict[Tuple[str, str], int] = {}
        for r, (a, b) in enumerate(merges):
            if a not in self.vocab or b not in self.vocab or (a + b) not in self.vocab:
                raise TokenizerError("merge refers to a token outside the vocabulary")
            if (a, b) in self.ranks:
                raise TokenizerError("duplicate merge")
            self.ranks[(a, b)] = r
        self.added = sorted(((s, i) for s, i in added), key=lambda x: (-len(x[0].encode()), x[1]))
        self.added_ids = {i for _, i in added}
        for s, i in added:
            self.id_to_token.setdefault(i, s)
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

    # ------------------------------------------------------------------ loading
    @classmethod
    def from_json(cls, text: str | bytes) -> "Tokenizer":
        raw = text.encode() if isinstance(text, str) else bytes(text)
        d = loads_strict(raw)
        if d.get("normalizer") is not None or d.get("post_processor") is not None:
            raise TokenizerError("normalizer and post_processor must be null")
        for key in ("pre_tokenizer", "decoder"):
            p = d.get(key)
            if not isinstance(p, dict) or p.get("type") != "ByteLevel" or p.get("use_regex", True) or \
                    p.get("add_prefix_space", False):
                raise TokenizerError(f"{key} must be ByteLevel without regex or prefix space")
        m = d.get("model")
        if not isinstance(m, dict) or m.get("type") != "BPE":
            raise TokenizerError("model must be BPE")
        for k in ("dropout", "unk_token", "continuing_subword_prefix", "end_of_word_suffix"):
            if m.get(k) is not None:
                raise TokenizerError(f"BPE {k} is not supported")
        for k in ("fuse_unk", "byte_fallback", "ignore_merges"):
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
        return cls(m["vocab"], merges, added, hashlib.sha256(raw).hexdigest())

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

    def encode_bytes(self, data: bytes, allow_special: bool = True) -> List[int]:
        if not self.added:
            return self._bpe(data)
        text = data
        ids: List[int] = []
        start = 0
        i = 0
        specials = [(s.encode(), t) for s, t in self.added]
        while i < len(text):
            hit = None
            for s, t in specials:
                if text.startswith(s, i):
                    hit = (s, t)
                    break
            if hit is None:
                i += 1
                continue
            if not allow_special:
                raise TokenizerError("input contains a special token")
            if start < i:
                ids += self._bpe(text[start:i])
            ids.append(hit[1])
            i += len(hit[0])
            start = i
        if start < len(text):
            ids += self._bpe(text[start:])
        return ids

    def encode(self, text: str, allow_special: bool = True) -> List[int]:
        return self.encode_bytes(text.encode("utf-8"), allow_special)

    # ------------------------------------------------------------------ decode
    def token_bytes(self, tid: int) -> bytes:
        t = self.id_to_token.get(tid)
        if t is None:
            raise TokenizerError("unknown token id")
        if tid in self.added_ids:
            return t.encode("utf-8")
        try:
            return bytes(_U2B[c] for c in t)
        except KeyError:
            raise TokenizerError("token outside the byte-level alphabet") from None

    def decode_bytes(self, ids: Iterable[int]) -> bytes:
        return b"".join(self.token_bytes(i) for i in ids)

    def decode(self, ids: Iterable[int]) -> str:
        return self.decode_bytes(ids).decode("utf-8", errors="replace")


def synthetic_byte_tokenizer(vocab_size: int = 256) -> Tokenizer:
    """A tokenizer whose ids 0..255 are the raw bytes (used with random-init
    models whose vocabulary has no text meaning)."""
    vocab = {_B2U[b]: b for b in range(256)}
    t = Tokenizer(vocab, [], digest=hashlib.sha256(b"lunaflux-byte-tokenizer").hexdigest())
    return t
