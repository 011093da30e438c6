"""ctypes binding for the CPU oracle (refcpu.c).

TEST INFRASTRUCTURE ONLY: tests/, __graft_entry__.smoke() and bench.py's
cpu_baseline / ``--impl reference`` legs use this as the checker or as the
timed CPU baseline. Nothing in the inferox_b200 package imports it.

Parity status: the Rust reference cannot be built on these machines (no
rustc/cargo), so this restatement is pinned by porting every known-answer
test the reference's sources hold (tests/test_oracle_kats.py); forward-pass
logits follow src/model/forward.rs line by line but no reference-generated
vector pins them.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_SO = os.path.join(_HERE, "_build", "librefcpu.so")

OK = 0
ERRORS = {
    1: "Io", 2: "InvalidMagic", 3: "UnsupportedVersion", 4: "UnknownValueType",
    5: "UnknownTensorType", 6: "InvalidUtf8", 7: "InvalidShape", 8: "UnexpectedEof",
    9: "TensorNotFound", 10: "InvalidTensorIndex", 11: "TensorOffsetOverflow",
    12: "UnsupportedArchitecture",
}

F32, F16, Q4_0, Q8_0, Q4_K, Q6_K, Q8_K, Q5_0 = 0, 1, 2, 7, 12, 14, 15, 5


class OracleError(RuntimeError):
    def __init__(self, code: int, what: str = ""):
        self.code = code
        self.name = ERRORS.get(code, f"code{code}")
        super().__init__(f"{what}: {self.name}" if what else self.name)


class RcConfig(C.Structure):
    _fields_ = [
        ("vocab_size", C.c_uint32),
        ("hidden_size", C.c_uint64), ("n_layers", C.c_uint64), ("n_heads", C.c_uint64),
        ("n_kv_heads", C.c_uint64), ("head_dim", C.c_uint64),
        ("intermediate_size", C.c_uint64),
        ("norm_eps", C.c_float), ("rope_base", C.c_float),
        ("rope_dim", C.c_uint64), ("context_length", C.c_uint64),
        ("architecture", C.c_char * 64),
    ]


class RcSynthSpec(C.Structure):
    _fields_ = [
        ("vocab", C.c_uint32), ("dim", C.c_uint32), ("n_layers", C.c_uint32),
        ("n_heads", C.c_uint32), ("n_kv_heads", C.c_uint32), ("ffn", C.c_uint32),
        ("context", C.c_uint32), ("rope_base", C.c_float), ("norm_eps", C.c_float),
        ("sigma", C.c_float), ("mix", C.c_int), ("tied", C.c_int), ("seed", C.c_uint64),
        ("threads", C.c_int),
    ]


# The benchmark's model shapes (the workload definition; mix 0 = all Q8_0,
# 1 = Q4_K_M). Kept beside the oracle so the reference arm needs nothing from
# the product package; a CPU test checks they equal the product's table.
BENCH_CONFIGS = {
    "tiny": dict(vocab=32000, dim=288, n_layers=6, n_heads=6, n_kv_heads=6, ffn=768, context=256,
                 rope_base=10000.0, mix=0, tied=0),
    "1b": dict(vocab=128256, dim=2048, n_layers=16, n_heads=32, n_kv_heads=8, ffn=8192,
               context=4096, rope_base=500000.0, mix=1, tied=1),
    "8b": dict(vocab=128256, dim=4096, n_layers=32, n_heads=32, n_kv_heads=8, ffn=14336,
               context=4096, rope_base=500000.0, mix=1, tied=0),
    "70b": dict(vocab=32000, dim=8192, n_layers=80, n_heads=64, n_kv_heads=8, ffn=28672,
                context=4096, rope_base=10000.0, mix=1, tied=0),
}


def build() -> str:
    """Compile the oracle with its Makefile (idempotent)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _SO


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_SO):
            build()
        L = C.CDLL(_SO)
        fp = C.POINTER(C.c_float)
        u8p = C.POINTER(C.c_uint8)
        u32p = C.POINTER(C.c_uint32)
        sz = C.c_size_t
        L.rc_f16_to_f32.restype = C.c_float
        L.rc_f16_to_f32.argtypes = [C.c_uint16]
        L.rc_type_byte_size.restype = C.c_int64
        L.rc_type_byte_size.argtypes = [C.c_int, C.c_uint64]
        L.rc_dequantize.argtypes = [C.c_int, u8p, sz, fp, sz]
        for name in ("rc_matmul", "rc_matmul_t", "rc_matmul_t_scalar_emul"):
            getattr(L, name).argtypes = [fp, fp, fp, sz, sz, sz]
        L.rc_rms_norm.argtypes = [fp, fp, sz, C.c_float]
        L.rc_rms_norm_rows.argtypes = [fp, fp, C.c_float, sz, sz]
        L.rc_silu.argtypes = [fp, sz]
        L.rc_swiglu.argtypes = [fp, fp, fp, sz]
        L.rc_add_in_place.argtypes = [fp, fp, sz]
        L.rc_softmax_rows.argtypes = [fp, sz, sz]
        L.rc_embedding_lookup.argtypes = [fp, sz, u32p, sz, sz, fp]
        L.rc_rope.argtypes = [fp, sz, sz, sz, sz, C.c_float]
        L.rc_argmax.restype = C.c_uint32
        L.rc_argmax.argtypes = [fp, sz]
        L.rc_sample.restype = C.c_uint32
        L.rc_sample.argtypes = [fp, sz, C.c_float, sz, C.c_float, C.c_double]
        L.rc_model_open_mem.argtypes = [u8p, sz, C.POINTER(C.c_void_p)]
        L.rc_model_free.argtypes = [C.c_void_p]
        L.rc_gguf_open_mem.argtypes = [u8p, sz, C.POINTER(C.c_void_p)]
        L.rc_tensor_bytes.argtypes = [C.c_void_p, C.c_char_p, C.POINTER(C.c_uint64),
                                      C.POINTER(C.c_uint64)]
        L.rc_model_config.argtypes = [C.c_void_p, C.POINTER(RcConfig)]
        L.rc_model_tensor_info.argtypes = [C.c_void_p, C.c_char_p, C.POINTER(C.c_int),
                                           C.POINTER(C.c_uint64), C.POINTER(C.c_uint64),
                                           C.POINTER(C.c_uint64)]
        L.rc_model_has_output.argtypes = [C.c_void_p]
        L.rc_model_n_tensors.argtypes = [C.c_void_p]
        L.rc_set_threads.argtypes = [C.c_int]
        L.rc_set_faithful.argtypes = [C.c_int]
        L.rc_kv_new.restype = C.c_void_p
        L.rc_kv_new.argtypes = [C.c_void_p, sz, sz]
        L.rc_kv_free.argtypes = [C.c_void_p]
        L.rc_kv_clear.argtypes = [C.c_void_p]
        L.rc_kv_len.restype = sz
        L.rc_kv_len.argtypes = [C.c_void_p]
        L.rc_kv_read.argtypes = [C.c_void_p, sz, C.c_int, fp]
        L.rc_prefill.argtypes = [C.c_void_p, C.c_void_p, u32p, sz, fp, C.c_int]
        L.rc_decode_step.argtypes = [C.c_void_p, C.c_void_p, C.c_uint32, fp]
        L.rc_forward.argtypes = [C.c_void_p, u32p, sz, fp]
        L.rc_generate.argtypes = [C.c_void_p, C.c_void_p, u32p, sz, sz, u32p]
        L.rc_synth_gguf.argtypes = [C.POINTER(RcSynthSpec), C.POINTER(C.POINTER(C.c_uint8)),
                                    C.POINTER(C.c_size_t)]
        L.rc_synth_free.argtypes = [C.POINTER(C.c_uint8)]
        _lib = L
    return _lib


def _f(a):
    return a.ctypes.data_as(C.POINTER(C.c_float))


def _u8(a):
    return a.ctypes.data_as(C.POINTER(C.c_uint8))


def _u32(a):
    return a.ctypes.data_as(C.POINTER(C.c_uint32))


def _chk(code, what=""):
    if code != OK:
        raise OracleError(code, what)


def f16_to_f32(h: int) -> float:
    return lib().rc_f16_to_f32(h)


def type_byte_size(ttype: int, n: int) -> int:
    return lib().rc_type_byte_size(ttype, n)


def dequantize(ttype: int, data: bytes | np.ndarray, n_out: int) -> np.ndarray:
    b = np.frombuffer(bytes(data), dtype=np.uint8) if not isinstance(data, np.ndarray) else data
    b = np.ascontiguousarray(b, dtype=np.uint8)
    out = np.zeros(n_out, dtype=np.float32)
    _chk(lib().rc_dequantize(ttype, _u8(b), b.size, _f(out), n_out), "dequantize")
    return out


def matmul_t(a, b, m, n, k, emul=False):
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    c = np.zeros(m * n, np.float32)
    fn = lib().rc_matmul_t_scalar_emul if emul else lib().rc_matmul_t
    fn(_f(a), _f(b), _f(c), m, n, k)
    return c


def matmul(a, b, m, n, k):
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    c = np.zeros(m * n, np.float32)
    lib().rc_matmul(_f(a), _f(b), _f(c), m, n, k)
    return c


def rms_norm(x, w, eps):
    x = np.array(x, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    lib().rc_rms_norm(_f(x), _f(w), x.size, eps)
    return x


def rms_norm_rows(x, w, eps, rows):
    x = np.array(x, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    lib().rc_rms_norm_rows(_f(x), _f(w), eps, rows, w.size)
    return x


def silu(x):
    x = np.array(x, np.float32)
    lib().rc_silu(_f(x), x.size)
    return x


def swiglu(g, u):
    g = np.ascontiguousarray(g, np.float32)
    u = np.ascontiguousarray(u, np.float32)
    o = np.zeros_like(g)
    lib().rc_swiglu(_f(g), _f(u), _f(o), g.size)
    return o


def add_in_place(o, b):
    o = np.array(o, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    lib().rc_add_in_place(_f(o), _f(b), o.size)
    return o


def softmax_rows(x, rows, cols):
    x = np.array(x, np.float32)
    lib().rc_softmax_rows(_f(x), rows, cols)
    return x


def embedding_lookup(emb, ids, hidden):
    emb = np.ascontiguousarray(emb, np.float32)
    ids = np.ascontiguousarray(ids, np.uint32)
    out = np.zeros(ids.size * hidden, np.float32)
    _chk(lib().rc_embedding_lookup(_f(emb), emb.size, _u32(ids), ids.size, hidden, _f(out)),
         "embedding_lookup")
    return out


def rope(x, seq, heads, hd, rope_dim, base):
    x = np.array(x, np.float32)
    lib().rc_rope(_f(x), seq, heads, hd, rope_dim, base)
    return x


def argmax(x):
    x = np.ascontiguousarray(x, np.float32)
    return int(lib().rc_argmax(_f(x), x.size))


def sample(logits, temperature, top_k, top_p, u):
    x = np.ascontiguousarray(logits, np.float32)
    return int(lib().rc_sample(_f(x), x.size, temperature, top_k, top_p, u))


def set_threads(n: int):
    lib().rc_set_threads(int(n))


def set_faithful(on: bool):
    lib().rc_set_faithful(1 if on else 0)


def synth_gguf(name: str | None = None, seed: int = 1234, threads: int = 0,
               **overrides) -> np.ndarray:
    """A benchmark model as a GGUF image (synth_ref.c), e.g. synth_gguf("8b")."""
    cfg = dict(BENCH_CONFIGS[name]) if name else {}
    cfg.update(overrides)
    sp = RcSynthSpec(vocab=cfg["vocab"], dim=cfg["dim"], n_layers=cfg["n_layers"],
                     n_heads=cfg["n_heads"], n_kv_heads=cfg["n_kv_heads"], ffn=cfg["ffn"],
                     context=cfg.get("context", 4096), rope_base=cfg.get("rope_base", 10000.0),
                     norm_eps=cfg.get("norm_eps", 1e-5), sigma=cfg.get("sigma", 0.02),
                     mix=cfg.get("mix", 1), tied=cfg.get("tied", 0), seed=seed,
                     threads=threads if threads > 0 else (os.cpu_count() or 1))
    p = C.POINTER(C.c_uint8)()
    n = C.c_size_t()
    _chk(lib().rc_synth_gguf(C.byref(sp), C.byref(p), C.byref(n)), "synth_gguf")
    try:
        out = np.empty(n.value, np.uint8)
        C.memmove(out.ctypes.data, p, n.value)
    finally:
        lib().rc_synth_free(p)
    return out


class GgufFile:
    """GgufFile::read + Weights::tensor over an in-memory image (file.rs:57-116,
    weights.rs:44-51)."""

    def __init__(self, data: bytes):
        self._buf = np.frombuffer(bytes(data), dtype=np.uint8).copy()
        h = C.c_void_p()
        _chk(lib().rc_gguf_open_mem(_u8(self._buf), self._buf.size, C.byref(h)), "GgufFile::read")
        self._h = h

    def __del__(self):
        h = getattr(self, "_h", None)
        if h is not None and h.value:
            lib().rc_model_free(h)
            self._h = None

    def n_tensors(self) -> int:
        return int(lib().rc_model_n_tensors(self._h))

    def tensor(self, name: str) -> bytes:
        off = C.c_uint64()
        nb = C.c_uint64()
        _chk(lib().rc_tensor_bytes(self._h, name.encode(), C.byref(off), C.byref(nb)), name)
        return self._buf[off.value:off.value + nb.value].tobytes()


class Model:
    """Model::open over an in-memory GGUF image (model/mod.rs:64-92)."""

    def __init__(self, data: bytes | np.ndarray):
        if isinstance(data, np.ndarray):
            self._buf = np.ascontiguousarray(data, np.uint8)
        else:
            self._buf = np.frombuffer(bytes(data), dtype=np.uint8).copy()
        h = C.c_void_p()
        _chk(lib().rc_model_open_mem(_u8(self._buf), self._buf.size, C.byref(h)), "Model::open")
        self._h = h
        c = RcConfig()
        lib().rc_model_config(h, C.byref(c))
        self.config = c

    @classmethod
    def open(cls, path: str) -> "Model":
        return cls(np.fromfile(path, dtype=np.uint8))

    def __del__(self):
        h = getattr(self, "_h", None)
        if h is not None and h.value:
            lib().rc_model_free(h)
            self._h = None

    @property
    def vocab(self) -> int:
        return int(self.config.vocab_size)

    def has_output(self) -> bool:
        return bool(lib().rc_model_has_output(self._h))

    def n_tensors(self) -> int:
        return int(lib().rc_model_n_tensors(self._h))

    def tensor_info(self, name: str):
        t = C.c_int()
        n = C.c_uint64()
        off = C.c_uint64()
        nb = C.c_uint64()
        _chk(lib().rc_model_tensor_info(self._h, name.encode(), C.byref(t), C.byref(n),
                                        C.byref(off), C.byref(nb)), name)
        return int(t.value), int(n.value), int(off.value), int(nb.value)

    def tensor_bytes(self, name: str) -> np.ndarray:
        _, _, off, nb = self.tensor_info(name)
        return self._buf[off:off + nb]

    def kv_cache(self, n_layers=None, max_seq=None) -> "KvCache":
        return KvCache(self, n_layers or int(self.config.n_layers),
                       max_seq or int(self.config.context_length))

    def prefill(self, ids, kv: "KvCache", last_row_only=False) -> np.ndarray:
        ids = np.ascontiguousarray(ids, np.uint32)
        rows = 1 if last_row_only else ids.size
        out = np.zeros(rows * self.vocab, np.float32)
        _chk(lib().rc_prefill(self._h, kv._h, _u32(ids), ids.size, _f(out),
                              1 if last_row_only else 0), "prefill")
        return out.reshape(rows, self.vocab)

    def decode_step(self, token: int, kv: "KvCache") -> np.ndarray:
        out = np.zeros(self.vocab, np.float32)
        _chk(lib().rc_decode_step(self._h, kv._h, int(token), _f(out)), "decode_step")
        return out

    def forward(self, ids) -> np.ndarray:
        ids = np.ascontiguousarray(ids, np.uint32)
        out = np.zeros(ids.size * self.vocab, np.float32)
        _chk(lib().rc_forward(self._h, _u32(ids), ids.size, _f(out)), "forward")
        return out.reshape(ids.size, self.vocab)

    def generate(self, prompt, max_tokens: int, kv: "KvCache") -> np.ndarray:
        p = np.ascontiguousarray(prompt, np.uint32)
        out = np.zeros(max_tokens, np.uint32)
        _chk(lib().rc_generate(self._h, kv._h, _u32(p), p.size, max_tokens, _u32(out)),
             "generate")
        return out


class KvCache:
    """KvCache (model/cache.rs:7-41)."""

    def __init__(self, model: Model, n_layers: int, max_seq: int):
        self._model = model
        self._h = C.c_void_p(lib().rc_kv_new(model._h, n_layers, max_seq))
        self.kv_dim = int(model.config.n_kv_heads * model.config.head_dim)

    def __del__(self):
        h = getattr(self, "_h", None)
        if h is not None and h.value:
            lib().rc_kv_free(h)
            self._h = None

    def clear(self):
        lib().rc_kv_clear(self._h)

    def __len__(self):
        return int(lib().rc_kv_len(self._h))

    def read(self, layer: int, which_v: bool) -> np.ndarray:
        n = len(self)
        out = np.zeros(n * self.kv_dim, np.float32)
        _chk(lib().rc_kv_read(self._h, layer, 1 if which_v else 0, _f(out)), "kv_read")
        return out.reshape(n, self.kv_dim)
