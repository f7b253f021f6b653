"""The GPT-2 tokenizer (tokenizer.mojo, host-side) against independent
implementations of the same pieces, on CPU:

- byte_to_codepoint equals bytes_to_unicode of Hugging Face transformers;
- pretokenize equals GPT-2's pre-tokenizer regex (the `regex` module) on the
  strings of the reference's tests/tokenizer_vs_tiktoken.py:16-25 and more;
- encode equals the `tokenizers` library's byte-level BPE (GPT-2's BPE model
  and ByteLevel pre-tokenizer) given the same vocab.json and merges.txt.

GPT-2's own vocab.json / merges.txt are not available here (no network), so
the BPE files are made by a small BPE trainer in this test from seeded text;
the comparison then checks the merge algorithm and the file reading, which is
what the reference's check against tiktoken exercises."""

import json
import random

import pytest

from llm_mojo_b200 import tokenizer as T

# the reference's own test strings (tests/tokenizer_vs_tiktoken.py:16-25)
REF_STRINGS = [
    "Hello, my name is",
    "The quick brown fox jumps over the lazy dog. It's 2026, isn't it? We'll see; they'd've known.",
    "  leading spaces\n\nand   multiple    spaces\tand tabs\n",
    "numbers 1234567 and 3.14159, emails a.b@c.com, URLs https://x.org/a?b=c",
    "Unicode: café naïve résumé — em dash “quotes” … 日本語 Привет мир 😀!",
    "CAPS'S and O'Neil's 'quoted' ''double''",
    "trailing spaces   ",
    "def f(x):\n    return x**2  # comment\n",
]
MORE = [
    "",
    " ",
    "a",
    "'s'S'd'll're've'm't",
    "x  \n\t y",
    "tabs\t\tand\r\nnewlines\n\n\n",
    "ÆØÅ æøå ß Ω ω",
]

GPT2_PATTERN = r"""'s|'t|'re|'ve|'m|'ll|'d| ?\p{L}+| ?\p{N}+| ?[^\s\p{L}\p{N}]+|\s+(?!\S)|\s+"""


def test_byte_to_codepoint_matches_transformers():
    from transformers.convert_slow_tokenizer import bytes_to_unicode

    ref = bytes_to_unicode()
    mine = T.byte_to_codepoint()
    assert [ord(ref[b]) for b in range(256)] == mine
    assert len(set(mine)) == 256


def _regex_chunks(s):
    import regex

    return [m.group(0) for m in regex.finditer(GPT2_PATTERN, s)]


def _my_chunks(s):
    b = s.encode("utf-8")
    out, start = [], 0
    for e in T.pretokenize(b):
        out.append(b[start:e].decode("utf-8"))
        start = e
    return out


@pytest.mark.parametrize("s", REF_STRINGS + MORE)
def test_pretokenize_matches_gpt2_regex(s):
    assert _my_chunks(s) == _regex_chunks(s)


def _train_bpe(texts, n_merges, seed):
    """A small byte-level BPE trainer: the most frequent adjacent pair within
    pre-tokenized chunks is merged, ties broken by a seeded order; returns
    (vocab: token string -> id, merges: [(a, b)])."""
    b2u = T.byte_to_codepoint()
    vocab = {chr(b2u[b]): i for i, b in enumerate(range(256))}
    words = []
    for s in texts:
        for w in _regex_chunks(s):
            words.append([chr(b2u[c]) for c in w.encode("utf-8")])
    rng = random.Random(seed)
    merges = []
    for _ in range(n_merges):
        counts = {}
        for w in words:
            for a, c in zip(w, w[1:]):
                counts[(a, c)] = counts.get((a, c), 0) + 1
        if not counts:
            break
        top = max(counts.values())
        cands = sorted(p for p, v in counts.items() if v == top)
        a, c = cands[rng.randrange(len(cands))]
        merges.append((a, c))
        if a + c not in vocab:
            vocab[a + c] = len(vocab)
        for w in words:
            i = 0
            while i < len(w) - 1:
                if w[i] == a and w[i + 1] == c:
                    w[i:i + 2] = [a + c]
                i += 1
    return vocab, merges


@pytest.fixture(scope="module")
def bpe_dir(tmp_path_factory):
    rng = random.Random(7)
    base = REF_STRINGS + MORE
    words = "the of and to in is it that was for on are with as his they be at one have this from".split()
    texts = base + [" ".join(rng.choice(words) for _ in range(40)) + "." for _ in range(30)]
    vocab, merges = _train_bpe(texts, 300, seed=3)
    d = tmp_path_factory.mktemp("bpe")
    with open(d / "vocab.json", "w", encoding="utf-8") as f:
        json.dump(vocab, f, ensure_ascii=False)
    with open(d / "merges.txt", "w", encoding="utf-8") as f:
        f.write("#version: 0.2\n")
        for a, c in merges:
            f.write(f"{a} {c}\n")
    return str(d)


def _hf_tokenizer(d):
    from tokenizers import Tokenizer, models, pre_tokenizers

    tok = Tokenizer(models.BPE.from_file(f"{d}/vocab.json", f"{d}/merges.txt"))
    tok.pre_tokenizer = pre_tokenizers.ByteLevel(add_prefix_space=False, use_regex=True)
    return tok


@pytest.mark.parametrize("s", REF_STRINGS + MORE + ["the of and to in is it that was for", "they have this one."])
def test_encode_matches_tokenizers_bpe(bpe_dir, s):
    mine = T.Tokenizer(bpe_dir)
    ref = _hf_tokenizer(bpe_dir)
    assert mine.encode(s) == ref.encode(s).ids
    assert mine.decode(mine.encode(s)) == s


def test_merges_are_used_and_ranked(bpe_dir):
    """Frequent words collapse to few tokens, and a pair's rank decides which
    merge applies first (the lowest rank wins among the chunk's pairs)."""
    tok = T.Tokenizer(bpe_dir)
    assert len(tok.encode(" the")) == 1
    assert len(tok.merges) > 100
    ranks = sorted(r >> 16 for r in tok.merges.values())
    assert ranks == list(range(len(ranks)))
    assert len(tok.token_bytes) >= T.VOCAB_SIZE
