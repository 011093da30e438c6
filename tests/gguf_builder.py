"""A GGUF writer for tests, mirroring the reference's test fixtures
(TestGgufBuilder, src/model/forward.rs:655-727; write_test_gguf,
src/gguf/weights.rs:121-149; write_test_llama_gguf, src/model/mod.rs:136-195).

Test infrastructure: it writes raw tensor bytes of any type with the same
header / metadata / tensor-info / 32-byte-aligned data layout the reference
parses (src/gguf/file.rs:57-116)."""
from __future__ import annotations

import struct

import numpy as np

U8, I8, U16, I16, U32, I32, F32V, BOOL, STR, ARR, U64, I64, F64 = range(13)


def _s(b: bytearray, s: str):
    e = s.encode()
    b += struct.pack("<Q", len(e)) + e


class GgufBuilder:
    def __init__(self, version: int = 3):
        self.version = version
        self.meta = bytearray()
        self.n_kv = 0
        self.tensors: list[tuple[str, list[int], int, bytes]] = []
        self.pad_between = True

    def u32(self, k, v):
        _s(self.meta, k); self.meta += struct.pack("<II", U32, v); self.n_kv += 1; return self

    def u64(self, k, v):
        _s(self.meta, k); self.meta += struct.pack("<IQ", U64, v); self.n_kv += 1; return self

    def f32(self, k, v):
        _s(self.meta, k); self.meta += struct.pack("<If", F32V, v); self.n_kv += 1; return self

    def string(self, k, v):
        _s(self.meta, k); self.meta += struct.pack("<I", STR); _s(self.meta, v); self.n_kv += 1
        return self

    def str_array(self, k, vals):
        _s(self.meta, k); self.meta += struct.pack("<IIQ", ARR, STR, len(vals))
        for v in vals:
            _s(self.meta, v)
        self.n_kv += 1
        return self

    def raw_kv(self, k, vt: int, payload: bytes):
        _s(self.meta, k); self.meta += struct.pack("<I", vt) + payload; self.n_kv += 1; return self

    def tensor(self, name, shape, ttype: int, data: bytes):
        self.tensors.append((name, list(shape), ttype, bytes(data)))
        return self

    def tensor_f32(self, name, shape, values):
        return self.tensor(name, shape, 0, np.asarray(values, np.float32).tobytes())

    def build(self) -> bytes:
        b = bytearray(b"GGUF")
        b += struct.pack("<IQQ", self.version, len(self.tensors), self.n_kv)
        b += self.meta
        offsets = []
        off = 0
        for _, _, _, data in self.tensors:
            offsets.append(off)
            off += len(data)
            if self.pad_between:
                off = (off + 31) // 32 * 32
        for (name, shape, ttype, _), o in zip(self.tensors, offsets):
            _s(b, name)
            b += struct.pack("<I", len(shape))
            for d in shape:
                b += struct.pack("<Q", d)
            b += struct.pack("<IQ", ttype, o)
        while len(b) % 32:
            b.append(0)
        base = len(b)
        for (_, _, _, data), o in zip(self.tensors, offsets):
            while len(b) < base + o:
                b.append(0)
            b += data
        return bytes(b)


def llama_meta(g: GgufBuilder, vocab, dim, layers, heads, kv_heads, ffn, ctx, eps=1e-5,
               rope_base=None):
    g.string("general.architecture", "llama")
    g.u32("llama.vocab_size", vocab)
    g.u32("llama.embedding_length", dim)
    g.u32("llama.block_count", layers)
    g.u32("llama.attention.head_count", heads)
    g.u32("llama.attention.head_count_kv", kv_heads)
    g.u32("llama.feed_forward_length", ffn)
    g.f32("llama.attention.layer_norm_rms_epsilon", eps)
    g.u32("llama.context_length", ctx)
    if rope_base is not None:
        g.f32("llama.rope.freq_base", rope_base)
    return g
