"""A byte-level BPE vocabulary for the tokenizer tests, trained here on generated text (test infrastructure).

The synthetic .qnt models carry a placeholder vocabulary (the 256 byte tokens, placeholders, the ChatML specials) with
no merges, which exercises nothing of BPE.  This module writes a tokenizer section with real merges and code-point
class ranges, in the .qnt layout (engine/src/model_file.cpp:172-187; scripts/export.py writes it): u32 count + (u32
length, bytes) per token, u32 count + (left, right, merged) per merge in priority order, u32 count + (id, length,
bytes) per special, then three lists of inclusive code-point ranges (letters, numbers, spaces).

Everything is generated from a fixed seed: the same vocabulary on every machine.
"""
from __future__ import annotations

import collections
import random
import re
import struct

SPECIALS = ["<|endoftext|>", "<|im_start|>", "<|im_end|>"]

# inclusive code-point ranges of the three classes beyond ASCII (a test stand-in for the Unicode tables)
LETTERS = [(0xAA, 0xAA), (0xB5, 0xB5), (0xBA, 0xBA), (0xC0, 0xD6), (0xD8, 0xF6), (0xF8, 0x2C1), (0x370, 0x373),
           (0x386, 0x3FF), (0x400, 0x481), (0x48A, 0x52F), (0x4E00, 0x9FFF), (0xAC00, 0xD7A3)]
NUMBERS = [(0xB2, 0xB3), (0xB9, 0xB9), (0xBC, 0xBE), (0x660, 0x669), (0x2160, 0x2188), (0xFF10, 0xFF19)]
SPACES = [(0x85, 0x85), (0xA0, 0xA0), (0x1680, 0x1680), (0x2000, 0x200A), (0x2028, 0x2029), (0x202F, 0x202F),
          (0x205F, 0x205F), (0x3000, 0x3000)]

_SYLLABLES = ["ka", "to", "re", "ven", "il", "mar", "qua", "nt", "sh", "or", "ed", "ing", "th", "ion", "al", "es",
              "pre", "fil", "ode", "cu", "da", "ker", "nel", "blo", "ck", "sca", "le", "head", "row", "ex", "act"]
_UNICODE_WORDS = ["café", "naïve", "Ωmega", "λόγος", "слово", "данные", "中文字符", "東京", "한국어", "façade", "Ärger",
                  "µs", "ºC"]
_PUNCT = [",", ".", "!", "?", ";", ":", "...", "--", "(", ")", "[", "]", "{", "}", "\"", "#", "$", "%", "&", "*", "+",
          "=", "/", "\\", "|", "@", "~", "`", "^", "<", ">", "™", "…", "—", "«", "»"]
_CONTRACTIONS = ["it's", "we're", "they've", "I'm", "you'll", "she'd", "don't", "IT'S", "We'Re", "o'clock", "rock'n'roll"]
_SPACES = [" ", "  ", "\t", "\n", "\r\n", "\n\n", " \n", " ", "　", " ", "   "]
_NUMBERS = ["7", "42", "2026", "3.14159", "1,024", "٣٤٥", "１２３", "²", "Ⅻ"]


def sample_text(rng: random.Random, n_words: int) -> str:
    """Generated prose mixing the classes the pre-tokenizer tells apart."""
    out = []
    for _ in range(n_words):
        r = rng.random()
        if r < 0.55:
            w = "".join(rng.choice(_SYLLABLES) for _ in range(rng.randint(1, 3)))
            out.append(w.capitalize() if rng.random() < 0.15 else w)
        elif r < 0.63:
            out.append(rng.choice(_UNICODE_WORDS))
        elif r < 0.70:
            out.append(rng.choice(_CONTRACTIONS))
        elif r < 0.78:
            out.append(rng.choice(_NUMBERS))
        else:
            out.append(rng.choice(_PUNCT))
        out.append(rng.choice(_SPACES) if rng.random() < 0.25 else " ")
    return "".join(out)


def train_merges(text: str, n_merges: int):
    """Byte-level BPE training: words (a space-led split) as byte-token tuples, the most frequent adjacent pair merged
    each round (ties to the smaller pair).  Returns the new tokens' bytes and the merges (left, right, merged)."""
    counts = collections.Counter(m.group(0).encode() for m in re.finditer(r" ?\S+|\s+", text))
    words = {tuple(w): c for w, c in counts.items()}
    pieces = [bytes([b]) for b in range(256)]
    merges = []
    for _ in range(n_merges):
        pairs = collections.Counter()
        for w, c in words.items():
            for a, b in zip(w, w[1:]):
                pairs[(a, b)] += c
        if not pairs:
            break
        (a, b), _ = min(pairs.items(), key=lambda kv: (-kv[1], kv[0]))
        new = len(pieces)
        pieces.append(pieces[a] + pieces[b])
        merges.append((a, b, new))
        nxt = {}
        for w, c in words.items():
            out, i = [], 0
            while i < len(w):
                if i + 1 < len(w) and w[i] == a and w[i + 1] == b:
                    out.append(new)
                    i += 2
                else:
                    out.append(w[i])
                    i += 1
            nxt[tuple(out)] = nxt.get(tuple(out), 0) + c
        words = nxt
    return pieces[256:], merges


def tokenizer_section(n_tokens: int, n_merges: int = 1200, seed: int = 2024) -> bytes:
    """The tokenizer section of a vocabulary of exactly n_tokens ids: bytes, merged tokens, unused placeholders, then
    the three specials at the end."""
    rng = random.Random(seed)
    text = sample_text(rng, 6000)
    n_merges = min(n_merges, n_tokens - 256 - len(SPECIALS))
    merged, merges = train_merges(text, n_merges)
    pieces = [bytes([b]) for b in range(256)] + merged
    while len(pieces) < n_tokens - len(SPECIALS):
        pieces.append(f"<unused{len(pieces)}>".encode())
    first_special = len(pieces)
    pieces += [s.encode() for s in SPECIALS]
    o = bytearray()
    o += struct.pack("<I", len(pieces))
    for p in pieces:
        o += struct.pack("<I", len(p)) + p
    o += struct.pack("<I", len(merges))
    for a, b, r in merges:
        o += struct.pack("<III", a, b, r)
    o += struct.pack("<I", len(SPECIALS))
    for i, s in enumerate(SPECIALS):
        o += struct.pack("<II", first_special + i, len(s.encode())) + s.encode()
    for table in (LETTERS, NUMBERS, SPACES):
        o += struct.pack("<I", len(table))
        for lo, hi in table:
            o += struct.pack("<II", lo, hi)
    return bytes(o)


def test_strings(rng: random.Random, n_fuzz: int):
    """Fixed cases around each rule of the split pattern, then generated ones."""
    fixed = [
        "", "a", " ", "  ", "\n", "hello world", "Hello, World!", "it's we're they've I'm you'll she'd",
        "IT'S SHE'LL 'S 'x ''", "  leading and trailing  ", "tabs\tand\u000bvertical\u000cfeed", "line\r\nbreak\n\n\nend",
        " \n \n  word", "x  \n", "numbers 1234567 and 3.14 and ٣٤٥ and １２３ ²", "punct!!! ?? ...\n\n next",
        " (parens) [brackets] {braces}", "café naïve Ωmega λόγος слово 中文字符 한국어", "mixed中文and English",
        "a b　c d", "emoji 😀 and 🚀!", "<|im_start|>user\nhi there<|im_end|>\n<|im_start|>assistant\n",
        "<|endoftext|><|endoftext|>", "<|im_st", "invalid \xff\xfe bytes", "trunc \xe4\xb8", "'''", "don't'n'roll",
        "ALLCAPS and MiXeD", "a1b2c3", "x" * 300, " " * 17 + "y", "\t\t\tz", "end with space ",
    ]
    out = [s.encode("latin-1") if "\xff" in s or "\xe4\xb8" in s else s.encode() for s in fixed]
    pool = (list("abcXYZ019 '\n\r\t.,!?-_") + ["é", "λ", "中", "٣", " ", "　", "😀", "'s", "'LL", "<|im_end|>"])
    for _ in range(n_fuzz):
        k = rng.randint(1, 40)
        s = "".join(rng.choice(pool) for _ in range(k))
        b = s.encode()
        if rng.random() < 0.15:  # a stray byte that is not UTF-8
            i = rng.randrange(len(b) + 1)
            b = b[:i] + bytes([rng.choice([0x80, 0xBF, 0xC3, 0xE4, 0xF0, 0xFF])]) + b[i:]
        out.append(b)
    return out
