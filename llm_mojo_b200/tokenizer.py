"""GPT-2 byte-level BPE tokenizer (tokenizer.mojo): the host side of text I/O.

Reads a Hugging Face vocab.json and merges.txt. `encode` splits the UTF-8
bytes with the hand-written GPT-2 pre-tokenizer (`pretokenize`,
tokenizer.mojo:224-282), maps each byte to its single-byte token and applies
BPE merges within each chunk (`Tokenizer.bpe`, tokenizer.mojo:180-207);
`decode` joins `token_bytes[id]`. The tokens feed `Model.generate` /
`llmq_generate` as ids; no GPU work is involved.
"""

from __future__ import annotations

import json
import os

VOCAB_SIZE = 50257  # tokenizer.mojo:11

LETTER, DIGIT, SPACE, OTHER = 0, 1, 2, 3  # tokenizer.mojo:66-69


def byte_to_codepoint() -> list[int]:
    """GPT-2's reversible byte -> printable-unicode mapping (bytes_to_unicode,
    tokenizer.mojo:30-45): printable bytes map to themselves, the others to
    256, 257, ... in byte order."""
    table = [0] * 256
    n = 0
    for b in range(256):
        printable = 33 <= b <= 126 or 161 <= b <= 172 or 174 <= b <= 255
        if printable:
            table[b] = b
        else:
            table[b] = 256 + n
            n += 1
    return table


def utf8_len(lead: int) -> int:
    """Bytes of the UTF-8 sequence led by `lead` (tokenizer.mojo:48-55)."""
    if lead < 0x80:
        return 1
    if lead < 0xE0:
        return 2
    if lead < 0xF0:
        return 3
    return 4


def decode_codepoint(b: bytes, i: int) -> int:
    """The code point at b[i] (tokenizer.mojo:58-64); a truncated sequence
    reads as its lead byte."""
    n = utf8_len(b[i])
    if n == 1 or i + n > len(b):
        return b[i]
    cp = b[i] & (0x7F >> n)
    for k in range(1, n):
        cp = (cp << 6) | (b[i + k] & 0x3F)
    return cp


def char_class(cp: int) -> int:
    """The \\p{L} / \\p{N} / \\s classes of GPT-2's pre-tokenizer regex, as
    tokenizer.mojo:72-96 approximates them for the scripts most text uses."""
    if 97 <= cp <= 122 or 65 <= cp <= 90:
        return LETTER
    if 48 <= cp <= 57:
        return DIGIT
    if cp == 32 or 9 <= cp <= 13 or cp == 0x85 or cp == 0xA0:
        return SPACE
    if 0x2000 <= cp <= 0x200A or cp == 0x2028 or cp == 0x2029:
        return SPACE
    if cp == 0x202F or cp == 0x205F or cp == 0x3000:
        return SPACE
    if cp < 0xAA:
        return OTHER
    if cp in (0xAA, 0xB5, 0xBA):
        return LETTER
    if 0xC0 <= cp <= 0x24F and cp not in (0xD7, 0xF7):
        return LETTER
    if 0x370 <= cp <= 0x1FFF:
        return LETTER  # Greek, Cyrillic, Hebrew, Arabic, Indic, ...
    if 0x3040 <= cp <= 0x9FFF:
        return LETTER  # kana, CJK
    if 0xAC00 <= cp <= 0xD7AF:
        return LETTER  # Hangul
    return OTHER


def class_at(b: bytes, k: int) -> int:
    return char_class(decode_codepoint(b, k))


def pretokenize(b: bytes) -> list[int]:
    """Splits UTF-8 bytes into chunks the way GPT-2's regex
    's|'t|'re|'ve|'m|'ll|'d| ?\\p{L}+| ?\\p{N}+| ?[^\\s\\p{L}\\p{N}]+|\\s+(?!\\S)|\\s+
    does (tokenizer.mojo:224-282). Returns the end offset of each chunk; BPE
    merges never cross chunks."""
    n = len(b)
    ends: list[int] = []
    i = 0
    while i < n:
        c0 = b[i]
        # contractions: 's 't 're 've 'm 'll 'd
        if c0 == ord("'") and i + 1 < n:
            c1 = b[i + 1]
            if c1 in (ord("s"), ord("t"), ord("m"), ord("d")):
                i += 2
                ends.append(i)
                continue
            if i + 2 < n:
                c2 = b[i + 2]
                if (c1, c2) in ((ord("r"), ord("e")), (ord("v"), ord("e")), (ord("l"), ord("l"))):
                    i += 3
                    ends.append(i)
                    continue
        # an optional leading space, then a run of letters, digits or symbols
        j = i
        if c0 == ord(" ") and i + 1 < n and class_at(b, i + 1) != SPACE:
            j = i + 1
        cls = class_at(b, j)
        if cls != SPACE:
            k = j + utf8_len(b[j])
            while k < n and class_at(b, k) == cls:
                k += utf8_len(b[k])
            ends.append(k)
            i = k
            continue
        # whitespace: \s+(?!\S) leaves the last space to prefix the next word
        k = i
        last = i
        count = 0
        while k < n and class_at(b, k) == SPACE:
            last = k
            k += utf8_len(b[k])
            count += 1
        i = last if (k < n and count > 1) else k
        ends.append(i)
    return ends


class Tokenizer:
    """Tokenizer (tokenizer.mojo:99-219): token_bytes[id] (raw bytes), byte_id[b]
    (the single-byte token of byte b), merges[(a << 16) | b] = (rank << 16) |
    merged id."""

    def __init__(self, directory: str):
        to_cp = byte_to_codepoint()
        from_cp = {cp: b for b, cp in enumerate(to_cp)}
        # vocab.json: {"<token>": id, ...}, the token text in bytes_to_unicode form
        with open(os.path.join(directory, "vocab.json"), encoding="utf-8") as f:
            vocab = json.load(f)
        size = max(VOCAB_SIZE, max(vocab.values()) + 1)
        self.ids: dict[str, int] = {}
        self.token_bytes: list[bytes] = [b""] * size
        for key, tid in vocab.items():
            self.ids[key] = tid
            self.token_bytes[tid] = bytes(from_cp[ord(ch)] for ch in key)
        self.byte_id = [self.ids[chr(to_cp[b])] for b in range(256)]
        # merges.txt: one "a b" pair per line, in priority order
        self.merges: dict[int, int] = {}
        with open(os.path.join(directory, "merges.txt"), encoding="utf-8") as f:
            text = f.read()
        rank = 0
        for line in text.split("\n"):
            if line.startswith("#version") or len(line) == 0:
                continue
            parts = line.split(" ")
            a, b = self.ids[parts[0]], self.ids[parts[1]]
            m = self.ids[parts[0] + parts[1]]
            self.merges[(a << 16) | b] = (rank << 16) | m
            rank += 1

    def bpe(self, toks: list[int]) -> list[int]:
        """Repeatedly merges every occurrence, left to right, of the adjacent
        pair with the lowest rank (tokenizer.mojo:180-207)."""
        while len(toks) > 1:
            best_rank, best_pair, best_id = None, -1, -1
            for i in range(len(toks) - 1):
                key = (toks[i] << 16) | toks[i + 1]
                r = self.merges.get(key)
                if r is not None and (best_rank is None or (r >> 16) < best_rank):
                    best_rank, best_id, best_pair = r >> 16, r & 0xFFFF, key
            if best_pair < 0:
                break
            merged: list[int] = []
            i = 0
            while i < len(toks):
                if i + 1 < len(toks) and ((toks[i] << 16) | toks[i + 1]) == best_pair:
                    merged.append(best_id)
                    i += 2
                else:
                    merged.append(toks[i])
                    i += 1
            toks = merged
        return toks

    def encode(self, text: str) -> list[int]:
        """Token ids of text (tokenizer.mojo:209-219)."""
        b = text.encode("utf-8")
        out: list[int] = []
        s = 0
        for e in pretokenize(b):
            out.extend(self.bpe([self.byte_id[b[k]] for k in range(s, e)]))
            s = e
        return out

    def decode_bytes(self, ids) -> bytes:
        """The raw bytes of ids (token_bytes[id] joined)."""
        return b"".join(self.token_bytes[int(i)] for i in ids)

    def decode(self, ids) -> str:
        """The text of ids; bytes that end inside a UTF-8 sequence become U+FFFD."""
        return self.decode_bytes(ids).decode("utf-8", errors="replace")
