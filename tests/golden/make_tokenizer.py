"""Writes tests/golden/tokenizer_small.json and tokenizer_cases.json.

The tokenizer is synthetic: a byte-level BPE (the GPT-2 byte alphabet of
src/tokenizer/bytes.rs, ids 3..258) with merges learned greedily on a
seeded corpus of made-up syllable words, plus three added tokens. The cases
are texts encoded and id lists decoded by the CPU restatement of the
reference tokenizer (oracle/tokenizer_ref.py), whose merge loop is the
reference's own quadratic procedure. Run from the repository root:

    python tests/golden/make_tokenizer.py
"""
from __future__ import annotations

import collections
import json
import os
import random
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from oracle.tokenizer_ref import BpeTokenizer, byte_encoder  # noqa: E402

SPECIAL = ["<|endoftext|>", "<|im_start|>", "<|im_end|>"]
N_MERGES = 400


def corpus(rng: random.Random, n_words: int) -> list[str]:
    onsets = ["", "b", "d", "f", "g", "k", "l", "m", "n", "p", "r", "s", "t", "v", "z", "sh", "tr", "kl"]
    vowels = ["a", "e", "i", "o", "u", "ai", "ou", "é", "ü"]
    codas = ["", "", "n", "r", "s", "l", "k", "st"]
    words = []
    for _ in range(n_words):
        w = "".join(rng.choice(onsets) + rng.choice(vowels) + rng.choice(codas)
                    for _ in range(rng.randint(1, 3)))
        words.append((" " if rng.random() < 0.8 else "") + w + rng.choice(["", "", "", ",", "."]))
    return words


def learn_merges(words: list[str], n: int) -> list[tuple[str, str]]:
    enc = byte_encoder()
    seqs = collections.Counter(tuple(enc[b] for b in w.encode()) for w in words)
    merges = []
    for _ in range(n):
        pairs = collections.Counter()
        for s, c in seqs.items():
            for a, b in zip(s, s[1:]):
                pairs[(a, b)] += c
        if not pairs:
            break
        (a, b), _ = max(pairs.items(), key=lambda kv: (kv[1], kv[0]))
        merges.append((a, b))
        new = collections.Counter()
        for s, c in seqs.items():
            out, i = [], 0
            while i < len(s):
                if i + 1 < len(s) and s[i] == a and s[i + 1] == b:
                    out.append(a + b)
                    i += 2
                else:
                    out.append(s[i])
                    i += 1
            new[tuple(out)] += c
        seqs = new
    return merges


def main() -> None:
    rng = random.Random(2024)
    words = corpus(rng, 6000)
    merges = learn_merges(words, N_MERGES)
    enc = byte_encoder()
    vocab = {s: i for i, s in enumerate(SPECIAL)}
    for b in range(256):
        vocab[enc[b]] = len(vocab)
    for a, b in merges:
        if a + b not in vocab:
            vocab[a + b] = len(vocab)
    doc = {
        "version": "1.0",
        "added_tokens": [{"id": vocab[s], "content": s, "special": True} for s in SPECIAL],
        "normalizer": None,
        "pre_tokenizer": None,
        "model": {"type": "BPE", "dropout": None, "unk_token": "<|endoftext|>",
                  "vocab": vocab, "merges": [f"{a} {b}" for a, b in merges]},
    }
    raw = json.dumps(doc, ensure_ascii=False, indent=None)
    with open(os.path.join(HERE, "tokenizer_small.json"), "w", encoding="utf-8") as f:
        f.write(raw)
    tok = BpeTokenizer.from_json(raw)
    texts = ["", "hello world", " ".join(w.strip() for w in corpus(rng, 40)),
             "<|im_start|>user" + "".join(corpus(rng, 12)) + "<|im_end|><|endoftext|>",
             "tab\tnew\nline  two  spaces", "ünïcödé — ✓ 漢字 🙂", "<|im_start|><|im_start|>x<|im_end",
             "".join(corpus(rng, 300))]
    cases = {"encode": [{"text": t, "ids": tok.encode(t)} for t in texts], "decode": []}
    V = len(vocab)
    for k in range(6):
        ids = [rng.randrange(V + 20) for _ in range(rng.randint(1, 40))]  # some unknown ids
        cases["decode"].append({"ids": ids, "text": tok.decode(ids)})
    # byte tokens that do not form UTF-8: lossy replacement
    cases["decode"].append({"ids": [vocab[enc[0xE2]], vocab[enc[0x82]], vocab["a"]],
                            "text": tok.decode([vocab[enc[0xE2]], vocab[enc[0x82]], vocab["a"]])})
    with open(os.path.join(HERE, "tokenizer_cases.json"), "w", encoding="utf-8") as f:
        json.dump(cases, f, ensure_ascii=False, indent=0)


if __name__ == "__main__":
    main()
