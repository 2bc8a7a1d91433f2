"""Synthetic tokenizer files for the public-API tests (engine/api/cachepotato.h: cp_open looks
for qwen2.5-tokenizer.bin and qwen2.5-unicode.bin next to the model).

The formats are the ones the reference's loaders read (engine/tokenizers/tokenizer.c:13-57,
tokenizer_qwen.c:33-50), written here from that description:
  CPT1  u32 magic "CPT1", u32 version 1, u32 n_vocab, u32 n_merges; per id a u16 length and the
        token's raw bytes; per merge (in rank order) u32 left id, u32 right id, u32 merged id
  UNI1  u32 magic "UNI1", u32 n; n sorted (lo, hi, class) code-point ranges, class 1 letter,
        2 number, anything outside the ranges is "other"
The vocabulary matches the synthetic model's (151,936 ids): the 256 single bytes, merged pieces
of common English letter pairs and words, filler tokens, and from id 151,643 the special tokens
(<|endoftext|>, <|im_start|>, <|im_end|>, then unique fillers), where the Qwen tokenizer looks
for them. Nothing here comes from a real tokenizer.
"""
from __future__ import annotations

import os
import struct

N_VOCAB = 151936
SPECIAL_FIRST = 151643
SPECIALS = [b"<|endoftext|>", b"<|im_start|>", b"<|im_end|>"]
TOK_FILE, UNI_FILE = "qwen2.5-tokenizer.bin", "qwen2.5-unicode.bin"

# merge steps in rank order: each joins two existing tokens' bytes
PAIRS = ["th", "he", "in", "er", "an", "re", "on", "at", "en", "nd", "es", "or", "te", "ed", "is", "it",
         "al", "ar", "st", "to", "ou", "le", "ve", "me", "hi", "ow", "ea", "ll", "lo", "wh", "el", " t",
         " a", " w", " h", " m", " i", " o", " s", "us", "ab", "ut", "ag", "ai", "ay"]
WORDS = ["the", " the", "her", "here", "hell", "hello", "ther", "there", "and", " and", "are", " are",
         "you", " you", "what", " what", "abo", "about", "wea", "weat", "weather", "ing", "tell", " tell",
         " me", " hi", " how", " is", "is", " it"]


def vocab_and_merges():
    vocab = [bytes([b]) for b in range(256)]
    index = {v: i for i, v in enumerate(vocab)}
    merges = []

    def add(piece: bytes):
        if piece in index:
            return
        # split into two existing tokens, the longest known prefix first
        for cut in range(len(piece) - 1, 0, -1):
            a, b = piece[:cut], piece[cut:]
            if a in index and b in index:
                merges.append((index[a], index[b], len(vocab)))
                index[piece] = len(vocab)
                vocab.append(piece)
                return
        raise ValueError(piece)

    for p in PAIRS:
        add(p.encode())
    for w in WORDS:
        add(w.encode())
    n_fill = SPECIAL_FIRST - len(vocab)
    vocab += [f"~{i:06d}".encode() for i in range(n_fill)]
    vocab += SPECIALS
    vocab += [f"<|extra_{i}|>".encode() for i in range(N_VOCAB - len(vocab))]
    assert len(vocab) == N_VOCAB and vocab[151645] == b"<|im_end|>"
    return vocab, merges


def write(dirpath: str) -> None:
    vocab, merges = vocab_and_merges()
    with open(os.path.join(dirpath, TOK_FILE), "wb") as f:
        f.write(struct.pack("<IIII", 0x31545043, 1, len(vocab), len(merges)))
        for v in vocab:
            f.write(struct.pack("<H", len(v)) + v)
        for a, b, o in merges:
            f.write(struct.pack("<III", a, b, o))
    ranges = [(ord("0"), ord("9"), 2), (ord("A"), ord("Z"), 1), (ord("a"), ord("z"), 1), (0xC0, 0x24F, 1)]
    with open(os.path.join(dirpath, UNI_FILE), "wb") as f:
        f.write(struct.pack("<II", 0x31494E55, len(ranges)))
        for lo, hi, c in ranges:
            f.write(struct.pack("<III", lo, hi, c))
