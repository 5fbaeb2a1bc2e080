"""Tokenizer parity with Hugging Face ``tokenizers`` (an implementation
independent of this repository) on trained byte-level BPE models in the
layouts of the Llama 3 and GPT-2 tokenizers: regex pre-tokenisation, ranked
merges, ``ignore_merges``, special tokens and a BOS template.

The reference compares its encoder with ``tokenizers`` 0.22.2 on a pinned
corpus (tests/reference_tokenizer/MANIFEST.md:1-45); here the tokenizer and
the expected ids are produced by ``tokenizers`` inside the test.
"""
import random

import pytest

tk = pytest.importorskip("tokenizers")

from lunaflux_b200.tokenizer.bpe import Tokenizer  # noqa: E402

# The pre-tokenisation pattern of the Llama 3 tokenizer.json.
LLAMA3_SPLIT = (r"(?i:'s|'t|'re|'ve|'m|'ll|'d)|[^\r\n\p{L}\p{N}]?\p{L}+|\p{N}{1,3}| ?[^\s\p{L}\p{N}]+[\r\n]*"
                r"|\s*[\r\n]+|\s+(?!\S)|\s+")
SPECIALS = ["<|begin_of_text|>", "<|end_of_text|>", "<|eot_id|>"]


def corpus(seed=0, n=3000):
    rnd = random.Random(seed)
    words = ["the", "model", "token", "serving", "Blackwell", "tensor", "über", "naïve", "東京", "данные",
             "it's", "we'll", "I'M", "don't", "12345", "3.14159", "x86_64", "  ", "\n", "\t", "🙂", "—", "--",
             "foo_bar", "CamelCase", "HTTP/1.1", "a+b=c", "(x)", "[y]", "{z}", "$100", "e-mail", "ÆØÅ"]
    out = []
    for _ in range(n):
        k = rnd.randint(3, 12)
        out.append(" ".join(rnd.choice(words) for _ in range(k)) + rnd.choice(["", ".", "!", "\n", "\n\n", "  "]))
    return out


def trained(layout: str, ignore_merges: bool) -> str:
    model = tk.models.BPE(ignore_merges=ignore_merges)
    t = tk.Tokenizer(model)
    if layout == "llama3":
        t.pre_tokenizer = tk.pre_tokenizers.Sequence([
            tk.pre_tokenizers.Split(tk.Regex(LLAMA3_SPLIT), behavior="isolated", invert=False),
            tk.pre_tokenizers.ByteLevel(add_prefix_space=False, use_regex=False)])
    else:
        t.pre_tokenizer = tk.pre_tokenizers.ByteLevel(add_prefix_space=False, use_regex=True)
    t.decoder = tk.decoders.ByteLevel()
    trainer = tk.trainers.BpeTrainer(vocab_size=700, special_tokens=SPECIALS,
                                     initial_alphabet=tk.pre_tokenizers.ByteLevel.alphabet(), show_progress=False)
    t.train_from_iterator(corpus(), trainer)
    if layout == "llama3":
        bos = t.token_to_id(SPECIALS[0])
        t.post_processor = tk.processors.Sequence([
            tk.processors.ByteLevel(trim_offsets=False),
            tk.processors.TemplateProcessing(single=f"{SPECIALS[0]} $A", special_tokens=[(SPECIALS[0], bos)])])
    return t.to_str()


CASES = ["", "hello world", "The model's tokens aren't cached.", "  leading and trailing  ", "tabs\tand\nnewlines\n\n",
         "numbers 1234567 and 3.14159 and 42", "東京 данные über naïve ÆØÅ", "emoji 🙂🙂 and — dashes --",
         "<|begin_of_text|>system<|eot_id|>user text<|end_of_text|>", "CamelCaseWords HTTP/1.1 a+b=c (x) [y] {z}",
         "I'M WE'LL DON'T it's", "\r\n\r\nwindows lines\r\n", "x" * 300, "serving serving serving",
         "unseen zqxj vwkp words", "a  b   c    d"]


@pytest.mark.parametrize("layout,ignore_merges", [("llama3", True), ("llama3", False), ("gpt2", False)])
def test_encode_matches_tokenizers(layout, ignore_merges):
    js = trained(layout, ignore_merges)
    ref = tk.Tokenizer.from_str(js)
    ours = Tokenizer.from_json(js)
    rnd = random.Random(1)
    texts = CASES + [" ".join(rnd.sample(corpus(seed=5, n=50), 3)) for _ in range(40)]
    for text in texts:
        for special in (False, True):
            want = ref.encode(text, add_special_tokens=special).ids
            got = ours.encode(text, add_special_tokens=special)
            assert got == want, (layout, text, special)
            assert ours.decode(got) == ref.decode(want, skip_special_tokens=False)
    if layout == "llama3":
        assert ours.bos_id == ref.token_to_id(SPECIALS[0])


def test_random_text_matches_tokenizers():
    """Random Unicode text (letters, digits, marks, whitespace runs, emoji,
    apostrophes) through both implementations, Llama 3 layout."""
    js = trained("llama3", True)
    ref = tk.Tokenizer.from_str(js)
    ours = Tokenizer.from_json(js)
    rnd = random.Random(11)
    alphabet = (list("abcxyzABCXYZ0123456789 \t\n\r'’.,;:!?-_()[]{}<>/\\\"") +
                ["é", "ß", "ñ", "東", "京", "д", "ы", "🙂", "👍🏽", "́", "​", "  ", "\n\n", "'s", "'LL"])
    for _ in range(300):
        text = "".join(rnd.choice(alphabet) for _ in range(rnd.randint(0, 60)))
        assert ours.encode(text) == ref.encode(text, add_special_tokens=False).ids, repr(text)
        assert ours.decode(ours.encode(text)) == text
