"""Host-side mirror of the reference's tokenizer API (src/tokenizer/mod.rs).

    tok = BpeTokenizer.from_file("tokenizer.json")   # mod.rs:61-64
    tok = BpeTokenizer.from_json(text)               # mod.rs:67-110
    ids = tok.encode("hello world")                  # mod.rs:194-204
    text = tok.decode(ids)                           # mod.rs:206-225

The work is done by the library (tokenizer.cpp behind ifx_tokenizer_*); a
failure raises IfxError named after the reference's TokenizerError variant
("Io", "Json", "UnsupportedModel").
"""
from __future__ import annotations

import ctypes as C

from ._lib import check, lib


class BpeTokenizer:
    """Byte-level BPE over a Hugging Face tokenizer.json."""

    def __init__(self, handle: int):
        self._h = C.c_void_p(handle)

    @classmethod
    def from_file(cls, path: str) -> "BpeTokenizer":
        h = C.c_void_p()
        check(lib.ifx_tokenizer_load(str(path).encode(), C.byref(h)), "BpeTokenizer::from_file")
        return cls(h.value)

    @classmethod
    def from_json(cls, raw: str | bytes) -> "BpeTokenizer":
        b = raw.encode() if isinstance(raw, str) else bytes(raw)
        h = C.c_void_p()
        check(lib.ifx_tokenizer_load_json(b, len(b), C.byref(h)), "BpeTokenizer::from_json")
        return cls(h.value)

    def encode(self, text: str | bytes) -> list[int]:
        b = text.encode() if isinstance(text, str) else bytes(text)
        n = C.c_size_t()
        cap = max(16, len(b) + 16)  # at most one id per byte, plus added tokens
        while True:
            buf = (C.c_uint32 * cap)()
            code = lib.ifx_tokenizer_encode(self._h, b, len(b), buf, cap, C.byref(n))
            if code == 20 and n.value > cap:  # Shape: grow to the reported count
                cap = n.value
                continue
            check(code, "Tokenizer::encode")
            return list(buf[: n.value])

    def decode(self, ids) -> str:
        ids = [int(i) for i in ids]
        arr = (C.c_uint32 * max(1, len(ids)))(*ids)
        n = C.c_size_t()
        cap = max(64, 8 * len(ids))
        while True:
            buf = C.create_string_buffer(cap)
            code = lib.ifx_tokenizer_decode(self._h, arr, len(ids), buf, cap, C.byref(n))
            if code == 20 and n.value > cap:
                cap = n.value
                continue
            check(code, "Tokenizer::decode")
            return buf.raw[: n.value].decode("utf-8")

    def vocab_size(self) -> int:
        n = C.c_size_t()
        check(lib.ifx_tokenizer_vocab_size(self._h, C.byref(n)))
        return n.value

    def close(self) -> None:
        if self._h and self._h.value:
            lib.ifx_tokenizer_free(self._h)
            self._h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
