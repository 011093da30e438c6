"""The library's BPE tokenizer (ifx_tokenizer_*) against the CPU restatement
of the reference's (oracle/tokenizer_ref.py), on CPU.

* The reference's own unit tests (src/tokenizer/mod.rs:271-317): the ASCII
  round trip through a 256-byte vocabulary with one merge, and an added
  token split out of the text. Both pin the oracle and the library.
* The committed fixtures (tests/golden/tokenizer_small.json and its cases).
* Seeded random vocabularies, merge lists and texts (Unicode, added tokens
  that overlap or share a prefix, unknown ids, bytes that are not UTF-8):
  encode and decode equal the oracle's exactly.
* The reference's error variants: Io, Json (malformed JSON, schema
  mismatches, the array form of merges), UnsupportedModel.
"""
import json
import os
import random
import time

import pytest

from inferox_b200 import IfxError
from inferox_b200.tokenizer import BpeTokenizer
from oracle import tokenizer_ref as T

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def tiny_tokenizer_json() -> str:
    """mod.rs:271-299: <|endoftext|> = 0, byte b = b + 1, one merge of two spaces."""
    enc = T.byte_encoder()
    vocab = {"<|endoftext|>": 0}
    for b in range(256):
        vocab[enc[b]] = b + 1
    space = enc[32]
    return json.dumps({"version": "1.0", "added_tokens": [{"content": "<|endoftext|>"}],
                       "model": {"type": "BPE", "vocab": vocab, "merges": [f"{space} {space}"],
                                 "unk_token": "<|endoftext|>"}})


@pytest.mark.parametrize("impl", ["library", "oracle"])
def test_reference_unit_tests(impl):
    raw = tiny_tokenizer_json()
    tok = BpeTokenizer.from_json(raw) if impl == "library" else T.BpeTokenizer.from_json(raw)
    ids = tok.encode("hello world")  # encode_decode_ascii_roundtrip (mod.rs:301-309)
    assert ids
    assert tok.decode(ids) == "hello world"
    assert 0 in tok.encode("hi<|endoftext|>lo")  # special_token_is_split (mod.rs:311-316)


def test_byte_tables():
    enc = T.byte_encoder()
    assert len(set(enc)) == 256
    assert all(enc[b] == chr(b) for b in range(0x21, 0x7F))
    assert enc[0] == "Ā" and enc[32] == "Ġ" and enc[0xAD] == "Ń"
    tok = BpeTokenizer.from_json(tiny_tokenizer_json())
    # every single-byte token decodes to its byte (a lone high byte is lossy)
    for b in range(128):
        assert tok.decode([b + 1]) == chr(b)
    assert tok.decode([0xE2 + 1, 0x82 + 1, 0xAC + 1]) == "€"


def test_golden_fixtures():
    raw = open(os.path.join(GOLDEN, "tokenizer_small.json"), encoding="utf-8").read()
    cases = json.load(open(os.path.join(GOLDEN, "tokenizer_cases.json"), encoding="utf-8"))
    lib_tok = BpeTokenizer.from_file(os.path.join(GOLDEN, "tokenizer_small.json"))
    ora_tok = T.BpeTokenizer.from_json(raw)
    for c in cases["encode"]:
        assert ora_tok.encode(c["text"]) == c["ids"]
        assert lib_tok.encode(c["text"]) == c["ids"], c["text"][:40]
        assert lib_tok.decode(c["ids"]) == c["text"]
    for c in cases["decode"]:
        assert lib_tok.decode(c["ids"]) == c["text"]
    assert lib_tok.vocab_size() == len(json.loads(raw)["model"]["vocab"])


def _random_tokenizer(rng: random.Random):
    enc = T.byte_encoder()
    alphabet = [enc[b] for b in range(256)]
    vocab, merges = {}, []
    specials = ["<s>", "</s>", "<s>x", "[X]", "ü"]  # "<s>" is a prefix of "<s>x"
    for s in specials:
        vocab[s] = len(vocab)
    for ch in alphabet:
        if rng.random() < 0.9:  # some bytes missing: those pieces become unk
            vocab[ch] = len(vocab)
    pieces = list(alphabet[:128]) + [enc[b] for b in "éü漢🙂".encode()]
    for _ in range(300):
        a, b = rng.choice(pieces), rng.choice(pieces)
        merges.append(f"{a} {b}")
        if rng.random() < 0.5:
            pieces.append(a + b)
        if rng.random() < 0.8:
            vocab.setdefault(a + b, len(vocab))
    merges.append(merges[3])  # a duplicate pair: the later rank wins
    merges.append("lonely")   # one part only: ignored
    merges.append(f"{enc[104]}　{enc[105]}")  # split on Unicode white space
    doc = {"added_tokens": [{"content": s, "id": vocab[s]} for s in specials],
           "model": {"type": "BPE", "vocab": vocab, "merges": merges, "unk_token": "[X]"}}
    return json.dumps(doc, ensure_ascii=rng.random() < 0.5), len(vocab)


def _random_text(rng: random.Random) -> str:
    parts = ["hi", "hello", " ", "  ", "ab", "<s>", "</s>", "<s>x", "[X]", "é", "ü", "漢字", "🙂",
             "\n", "\t", "qq", "zz", "<s", "x</s"]
    return "".join(rng.choice(parts) for _ in range(rng.randint(0, 30)))


@pytest.mark.parametrize("seed", range(6))
def test_random_parity(seed):
    rng = random.Random(seed)
    raw, V = _random_tokenizer(rng)
    lib_tok, ora_tok = BpeTokenizer.from_json(raw), T.BpeTokenizer.from_json(raw)
    for _ in range(60):
        text = _random_text(rng)
        ids = ora_tok.encode(text)
        assert lib_tok.encode(text) == ids, text
        assert lib_tok.decode(ids) == ora_tok.decode(ids)
    for _ in range(60):
        ids = [rng.randrange(V + 10) for _ in range(rng.randint(0, 25))]
        assert lib_tok.decode(ids) == ora_tok.decode(ids), ids


def test_long_piece():
    # one piece of 6k bytes (the reference has no pre-tokenizer): the heap
    # merge gives the quadratic loop's result and stays fast
    raw = open(os.path.join(GOLDEN, "tokenizer_small.json"), encoding="utf-8").read()
    lib_tok, ora_tok = BpeTokenizer.from_json(raw), T.BpeTokenizer.from_json(raw)
    rng = random.Random(7)
    text = "".join(rng.choice(["tra", "ou", " kl", "é", "st", "ai", " "]) for _ in range(3000))
    t0 = time.perf_counter()
    ids = lib_tok.encode(text * 20)
    assert time.perf_counter() - t0 < 5.0
    assert lib_tok.encode(text) == ora_tok.encode(text)
    assert lib_tok.decode(ids) == text * 20


def test_buffer_sizing_and_empty():
    import ctypes as C

    from inferox_b200 import _lib
    tok = BpeTokenizer.from_json(tiny_tokenizer_json())
    n = C.c_size_t()
    code = _lib.lib.ifx_tokenizer_encode(tok._h, b"hello", 5, None, 0, C.byref(n))
    assert code == 20 and n.value == 5  # Shape, with the count a buffer needs
    assert tok.encode("") == [] and tok.decode([]) == ""


def _err(raw):
    with pytest.raises(IfxError) as e:
        BpeTokenizer.from_json(raw)
    return e.value.name


def test_errors(tmp_path):
    good = json.loads(tiny_tokenizer_json())
    assert _err("{") == "Json"
    assert _err(tiny_tokenizer_json() + " x") == "Json"  # trailing characters
    assert _err('{"model": {"type": "BPE", "vocab": {}}}') == "Json"  # no merges
    assert _err('{"added_tokens": [], "model": {"type": "BPE", "vocab": {}, "merges": [["a", "b"]]}}') == "Json"
    assert _err('{"model": {"type": "BPE", "vocab": {"a": 1.0}, "merges": []}}') == "Json"
    assert _err('{"model": {"type": "BPE", "vocab": {"a": -1}, "merges": []}}') == "Json"
    assert _err('{"model": {"type": "BPE", "vocab": {"a": 4294967296}, "merges": []}}') == "Json"
    assert _err('{"model": {"type": "BPE", "type": "BPE", "vocab": {}, "merges": []}}') == "Json"
    assert _err('{"added_tokens": [{"id": 1}], "model": {"type": "BPE", "vocab": {}, "merges": []}}') == "Json"
    assert _err('{"model": {"type": "BPE", "vocab": {"\\ud800": 1}, "merges": []}}') == "Json"
    # a schema error comes before the model-type check (mod.rs:69-73)
    assert _err('{"model": {"type": "WordPiece", "vocab": {}}}') == "Json"
    assert _err('{"model": {"type": "WordPiece", "vocab": {}, "merges": []}}') == "UnsupportedModel"
    # unknown fields and a null unk_token are accepted; unk_id then is 0
    ok = BpeTokenizer.from_json('{"x": [1, {"y": null}], "model": {"type": "BPE", "vocab": {"a": 5}, '
                                '"merges": [], "unk_token": null, "dropout": null}}')
    assert ok.encode("ab") == [5, 0]
    with pytest.raises(IfxError) as e:
        BpeTokenizer.from_file(str(tmp_path / "missing.json"))
    assert e.value.name == "Io"
    bad = tmp_path / "bad.json"
    bad.write_bytes(json.dumps(good).encode()[:-1] + b"\xff}")
    with pytest.raises(IfxError) as e:
        BpeTokenizer.from_file(str(bad))
    assert e.value.name == "Io"  # read_to_string: not UTF-8
    for impl in (BpeTokenizer, T.BpeTokenizer):  # both reject the same inputs
        with pytest.raises(Exception):
            impl.from_json('{"model": {"type": "BPE", "vocab": {}, "merges": [1]}}')
