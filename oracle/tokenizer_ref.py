"""CPU restatement of the reference's byte-level BPE tokenizer (test
infrastructure: the checker for tokenizer.cpp, never on the product path).

Follows src/tokenizer/mod.rs and bytes.rs step by step, including the
quadratic merge loop (mod.rs:114-140: rescan every adjacent pair, merge the
lowest rank, leftmost among equals), so the library's heap-based merge
order is checked against the reference's own procedure. Pinned by the
reference's two unit tests (mod.rs:271-317: the ASCII round trip through a
256-byte vocabulary with one merge, and an added token split out of the
text), restated in tests/test_tokenizer.py.

Where the reference is not deterministic (two added tokens at the same
position: HashSet order; an id shared by two vocabulary entries: HashMap
order), this restatement makes the same choice as the library (the longer
token; the later entry in the file), which is one of the reference's
possible outcomes.
"""
from __future__ import annotations

import json


def byte_encoder() -> list[str]:
    """bytes.rs:10-27."""
    out, n = [], 0
    for b in range(256):
        if 0x21 <= b <= 0x7E or 0xA1 <= b <= 0xAC or 0xAE <= b <= 0xFF:
            out.append(chr(b))
        else:
            out.append(chr(0x100 + n))
            n += 1
    return out


def byte_decoder() -> dict[str, int]:
    """bytes.rs:30-35."""
    return {c: i for i, c in enumerate(byte_encoder())}


class TokenizerError(Exception):
    def __init__(self, kind: str, msg: str):
        self.kind = kind
        super().__init__(f"{kind}: {msg}")


class BpeTokenizer:
    @classmethod
    def from_json(cls, raw: str) -> "BpeTokenizer":
        """mod.rs:67-110."""
        try:
            parsed = json.loads(raw)
        except ValueError as e:
            raise TokenizerError("Json", str(e))
        if not isinstance(parsed, dict) or not isinstance(parsed.get("model"), dict):
            raise TokenizerError("Json", "model")
        m = parsed["model"]
        for k in ("type", "vocab", "merges"):
            if k not in m:
                raise TokenizerError("Json", f"missing field `{k}`")
        if not isinstance(m["type"], str) or not isinstance(m["vocab"], dict) \
                or not isinstance(m["merges"], list) or not all(isinstance(x, str) for x in m["merges"]):
            raise TokenizerError("Json", "invalid type")
        for v in m["vocab"].values():
            if isinstance(v, bool) or not isinstance(v, int) or not 0 <= v <= 0xFFFFFFFF:
                raise TokenizerError("Json", "vocab value")
        added = parsed.get("added_tokens", [])
        if not isinstance(added, list) or not all(isinstance(t, dict) and isinstance(t.get("content"), str)
                                                  for t in added):
            raise TokenizerError("Json", "added_tokens")
        unk = m.get("unk_token")
        if unk is not None and not isinstance(unk, str):
            raise TokenizerError("Json", "unk_token")
        if m["type"] != "BPE":
            raise TokenizerError("UnsupportedModel", m["type"])
        t = cls()
        t.vocab = dict(m["vocab"])
        t.id_to_token = {}
        for tok, i in t.vocab.items():  # dict order: file order, later duplicates win
            t.id_to_token[i] = tok
        t.merges = {}
        for rank, line in enumerate(m["merges"]):
            parts = line.split()  # str.split() splits on Unicode white space too
            a = parts[0] if len(parts) > 0 else ""
            b = parts[1] if len(parts) > 1 else ""
            if a and b:
                t.merges[(a, b)] = rank
        t.special = []
        for tok in added:
            if tok["content"] not in t.special:
                t.special.append(tok["content"])
        t.unk_id = t.vocab.get(unk, 0) if unk is not None else 0
        return t

    def bpe(self, pieces: list[str]) -> list[str]:
        """mod.rs:114-140, literally."""
        if len(pieces) < 2:
            return pieces
        while True:
            best_rank, best_idx = None, 0
            for i in range(len(pieces) - 1):
                r = self.merges.get((pieces[i], pieces[i + 1]))
                if r is not None and (best_rank is None or r < best_rank):
                    best_rank, best_idx = r, i
            if best_rank is None:
                return pieces
            pieces[best_idx] = pieces[best_idx] + pieces[best_idx + 1]
            del pieces[best_idx + 1]

    def encode_piece(self, text: str) -> list[int]:
        """mod.rs:142-155."""
        enc = byte_encoder()
        merged = self.bpe([enc[b] for b in text.encode()])
        return [self.vocab.get(s, self.unk_id) for s in merged]

    def split_special(self, text: str) -> list[str]:
        """mod.rs:157-191 (ties at one position: the longer token)."""
        if not self.special:
            return [text]
        out, rem = [], text
        while rem:
            found = None
            for tok in self.special:
                if not tok:
                    continue
                p = rem.find(tok)
                if p >= 0 and (found is None or p < found[0] or (p == found[0] and len(tok) > len(found[1]))):
                    found = (p, tok)
            if found is None:
                out.append(rem)
                break
            p, tok = found
            if p > 0:
                out.append(rem[:p])
            out.append(tok)
            rem = rem[p + len(tok):]
        return out

    def encode(self, text: str) -> list[int]:
        """mod.rs:194-204."""
        ids = []
        for piece in self.split_special(text):
            if piece in self.special:
                ids.append(self.vocab.get(piece, self.unk_id))
            else:
                ids.extend(self.encode_piece(piece))
        return ids

    def decode(self, tokens) -> str:
        """mod.rs:206-225; String::from_utf8_lossy is bytes.decode(errors="replace")
        (both replace each maximal invalid subsequence with one U+FFFD)."""
        dec = byte_decoder()
        out = bytearray()
        for i in tokens:
            tok = self.id_to_token.get(int(i))
            if tok is None:
                continue
            for ch in tok:
                if ch in dec:
                    out.append(dec[ch])
                else:
                    out.extend(ch.encode())
        return out.decode("utf-8", errors="replace")
