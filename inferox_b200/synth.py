"""Synthetic benchmark models (the configurations of the reference's
workloads with seeded N(0, 0.02) weights), built by the C ABI's generator.

CONFIGS holds the four model shapes; `build(name)` returns a GGUF image as a
numpy uint8 array (host memory).
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from ._lib import SynthSpec, check, lib

# mix: 0 = all Q8_0, 1 = Q4_K_M (Q6_K for attn_v, even-layer ffn_down, output)
CONFIGS = {
    "tiny": dict(vocab=32000, dim=288, n_layers=6, n_heads=6, n_kv_heads=6, ffn=768, context=256,
                 rope_base=10000.0, mix=0, tied=0),
    "1b": dict(vocab=128256, dim=2048, n_layers=16, n_heads=32, n_kv_heads=8, ffn=8192,
               context=4096, rope_base=500000.0, mix=1, tied=1),
    "8b": dict(vocab=128256, dim=4096, n_layers=32, n_heads=32, n_kv_heads=8, ffn=14336,
               context=4096, rope_base=500000.0, mix=1, tied=0),
    "70b": dict(vocab=32000, dim=8192, n_layers=80, n_heads=64, n_kv_heads=8, ffn=28672,
                context=4096, rope_base=10000.0, mix=1, tied=0),
}


def spec(name: str | None = None, seed: int = 1234, threads: int = 0, **overrides) -> SynthSpec:
    cfg = dict(CONFIGS[name]) if name else {}
    cfg.update(overrides)
    s = SynthSpec()
    s.vocab = cfg["vocab"]
    s.dim = cfg["dim"]
    s.n_layers = cfg["n_layers"]
    s.n_heads = cfg["n_heads"]
    s.n_kv_heads = cfg["n_kv_heads"]
    s.ffn = cfg["ffn"]
    s.context = cfg.get("context", 4096)
    s.rope_base = cfg.get("rope_base", 10000.0)
    s.norm_eps = cfg.get("norm_eps", 1e-5)
    s.sigma = cfg.get("sigma", 0.02)
    s.mix = cfg.get("mix", 1)
    s.tied = cfg.get("tied", 0)
    s.seed = seed
    s.threads = threads
    return s


def build(name: str | None = None, seed: int = 1234, threads: int = 0, **overrides) -> np.ndarray:
    s = spec(name, seed, threads, **overrides)
    p = C.c_void_p()
    n = C.c_size_t()
    check(lib.ifx_synth_gguf(C.byref(s), C.byref(p), C.byref(n)), "synth_gguf")
    try:
        out = np.empty(n.value, np.uint8)
        C.memmove(out.ctypes.data, p, n.value)
    finally:
        lib.ifx_synth_free(p)
    return out


def quantize(ttype: int, x: np.ndarray) -> bytes:
    x = np.ascontiguousarray(x, np.float32)
    blk = {2: (32, 18), 7: (32, 34), 12: (256, 144), 14: (256, 210)}[ttype]
    out = np.empty(x.size // blk[0] * blk[1], np.uint8)
    check(lib.ifx_quantize(ttype, x.ctypes.data_as(C.c_void_p), x.size,
                           out.ctypes.data_as(C.c_void_p)), "quantize")
    return out.tobytes()


def normal(seed: int, stream: int, sigma: float, n: int) -> np.ndarray:
    out = np.empty(n, np.float32)
    check(lib.ifx_synth_normal(seed, stream, sigma, out.ctypes.data_as(C.POINTER(C.c_float)), n),
          "synth_normal")
    return out


def prompt_ids(vocab: int, n: int, seq_index: int = 0, seed: int = 42) -> np.ndarray:
    """Seeded uniform token ids in [3, vocab) (seed 42 + sequence index)."""
    rng = np.random.default_rng(seed + seq_index)
    return rng.integers(3, vocab, size=n, dtype=np.uint32)
