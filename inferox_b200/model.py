"""Host-side mirror of the reference's model API (src/model/mod.rs,
src/model/forward.rs, src/model/cache.rs, src/sampler.rs) over the C ABI.

    model = Model.open("model.gguf")              # Model::open
    kv = model.kv_cache(max_seq)                   # KvCache::new
    logits = model.prefill(ids, kv)                # Model::prefill
    logits = model.decode_step(token, kv)          # Model::decode_step
    tokens = model.generate(prompt, n, kv)         # Model::generate (greedy)
    tok = Sampler(0.8, 40, 0.95).sample(model)     # Sampler::sample on device

Errors raise IfxError whose `.name` is the gguf::Error variant
(src/gguf/error.rs:6-42) or one of the GPU build's additions.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np

from ._lib import Config, IfxError, LoadOpts, SamplerC, check, lib


def _u32(a):
    return a.ctypes.data_as(C.POINTER(C.c_uint32))


def _f32(a):
    return a.ctypes.data_as(C.POINTER(C.c_float))


def load_opts(device: int = 0, rope_compat: bool = True, use_graphs: bool = True,
              tp_size: int = 1, tp_rank: int = 0, nccl_comm: int | None = None,
              persistent_decode: bool = True, kquant_layout: str = "reference",
              tp_timeout_ms: int = 0) -> LoadOpts:
    """ifx_load_opts; kquant_layout "reference" reads type ids and Q4_K/Q6_K
    bytes as the reference does, "ggml" reads a file written by llama.cpp."""
    o = LoadOpts()
    lib.ifx_load_opts_default(C.byref(o))
    o.device = device
    o.rope_compat = 1 if rope_compat else 0
    o.use_graphs = 1 if use_graphs else 0
    o.tp_size = tp_size
    o.tp_rank = tp_rank
    o.nccl_comm = nccl_comm
    o.persistent_decode = 1 if persistent_decode else 0
    if kquant_layout not in ("reference", "ggml"):
        raise ValueError(f"kquant_layout must be 'reference' or 'ggml', not {kquant_layout!r}")
    o.kquant_layout = 1 if kquant_layout == "ggml" else 0
    o.tp_timeout_ms = tp_timeout_ms
    return o


class Model:
    """A model resident on one GPU (weights uploaded and repacked once)."""

    def __init__(self, handle: C.c_void_p):
        self._h = handle
        c = Config()
        check(lib.ifx_model_config(self._h, C.byref(c)), "model_config")
        self.config = c

    @classmethod
    def open(cls, path: str, **opts) -> "Model":
        h = C.c_void_p()
        o = load_opts(**opts)
        check(lib.ifx_model_load(path.encode(), C.byref(o), C.byref(h)), "Model::open")
        return cls(h)

    @classmethod
    def from_bytes(cls, data, **opts) -> "Model":
        buf = np.frombuffer(data, dtype=np.uint8) if not isinstance(data, np.ndarray) else data
        h = C.c_void_p()
        o = load_opts(**opts)
        check(lib.ifx_model_load_mem(buf.ctypes.data_as(C.c_void_p), buf.nbytes, C.byref(o),
                                     C.byref(h)), "Model::open")
        return cls(h)

    def close(self):
        if getattr(self, "_h", None) is not None and self._h.value:
            lib.ifx_model_free(self._h)
            self._h = None

    def __del__(self):
        self.close()

    @property
    def vocab(self) -> int:
        return int(self.config.vocab_size)

    def decode_weight_bytes(self) -> int:
        return int(lib.ifx_model_decode_weight_bytes(self._h))

    def kv_cache(self, max_seq: int | None = None) -> "KvCache":
        return KvCache(self, max_seq or int(self.config.context_length))

    def kv_batch(self, batch: int, max_seq: int | None = None, pages: int = 0) -> "KvBatch":
        """`batch` independent sequences decoded together (one weight read per
        step). pages > 0: the caches share a pool of that many 64-position
        pages, taken as sequences grow and returned by reset()."""
        return KvBatch(self, batch, max_seq or int(self.config.context_length), pages)

    def prefill(self, ids, kv: "KvCache", last_row_only: bool = False) -> np.ndarray:
        ids = np.ascontiguousarray(ids, np.uint32)
        rows = 1 if last_row_only else ids.size
        out = np.empty(rows * self.vocab, np.float32)
        check(lib.ifx_prefill(self._h, kv._h, _u32(ids), ids.size, _f32(out),
                              1 if last_row_only else 0), "prefill")
        return out.reshape(rows, self.vocab)

    def forward(self, ids, last_row_only: bool = False) -> np.ndarray:
        """Model::forward / forward_last_token_logits: full attention, no cache."""
        ids = np.ascontiguousarray(ids, np.uint32)
        rows = 1 if last_row_only else ids.size
        out = np.empty(rows * self.vocab, np.float32)
        check(lib.ifx_forward(self._h, _u32(ids), ids.size, _f32(out), 1 if last_row_only else 0),
              "forward")
        return out.reshape(rows, self.vocab)

    def decode_step(self, token: int, kv: "KvCache", want_logits: bool = True):
        out = np.empty(self.vocab, np.float32) if want_logits else None
        check(lib.ifx_decode_step(self._h, kv._h, int(token),
                                  _f32(out) if want_logits else None), "decode_step")
        return out

    def decode_greedy(self, token: int, n_steps: int, kv: "KvCache", timed: bool = False):
        """n_steps greedy steps fed on the device; returns (tokens, device_ms)."""
        out = np.empty(max(n_steps, 1), np.uint32)
        ms = C.c_float(0.0)
        check(lib.ifx_decode_greedy(self._h, kv._h, int(token), n_steps, _u32(out),
                                    C.byref(ms) if timed else None), "decode_greedy")
        return out[:n_steps], (float(ms.value) if timed else None)

    def bench_kernel(self, kv: "KvCache", which: str, reps: int):
        """(ms per launch, algorithmic bytes per launch) of one fused kernel."""
        ms = C.c_float(0.0)
        b = C.c_uint64(0)
        check(lib.ifx_bench_kernel(self._h, kv._h, which.encode(), reps, C.byref(ms), C.byref(b)),
              "bench_kernel")
        return float(ms.value), int(b.value)

    def generate(self, prompt, max_tokens: int, kv: "KvCache") -> np.ndarray:
        p = np.ascontiguousarray(prompt, np.uint32)
        out = np.empty(max(max_tokens, 1), np.uint32)
        check(lib.ifx_generate(self._h, kv._h, _u32(p), p.size, max_tokens, _u32(out)),
              "generate")
        return out[:max_tokens]


class KvCache:
    """Device-resident KV cache (f16, [layer][kv_head][max_seq][head_dim])."""

    def __init__(self, model: Model, max_seq: int):
        self._model = model
        h = C.c_void_p()
        check(lib.ifx_kv_create(model._h, max_seq, C.byref(h)), "KvCache::new")
        self._h = h
        self.max_seq = max_seq
        self.kv_dim = int(model.config.n_kv_heads * model.config.head_dim)

    def close(self):
        if getattr(self, "_h", None) is not None and self._h.value:
            lib.ifx_kv_free(self._h)
            self._h = None

    def __del__(self):
        self.close()

    def clear(self):
        check(lib.ifx_kv_clear(self._h), "KvCache::clear")

    def __len__(self) -> int:
        return int(lib.ifx_kv_len(self._h))

    def decode_kernels(self) -> int:
        """Kernels one decode step launches on this cache (1: persistent kernel)."""
        return int(lib.ifx_kv_decode_kernels(self._h))

    def read(self, layer: int, which_v: bool) -> np.ndarray:
        n = len(self)
        out = np.empty(max(n * self.kv_dim, 1), np.float32)
        check(lib.ifx_kv_read(self._h, layer, 1 if which_v else 0, _f32(out)), "kv_read")
        return out[: n * self.kv_dim].reshape(n, self.kv_dim)


class KvBatch:
    """`batch` KV caches decoded together: prefill each sequence, then step all."""

    PAGE_ROWS = 64

    def __init__(self, model: Model, batch: int, max_seq: int, pages: int = 0):
        self._model = model
        h = C.c_void_p()
        if pages:
            check(lib.ifx_kv_batch_create_paged(model._h, max_seq, batch, pages, C.byref(h)),
                  "kv_batch_create_paged")
        else:
            check(lib.ifx_kv_batch_create(model._h, max_seq, batch, C.byref(h)), "kv_batch_create")
        self._h = h
        self.batch, self.max_seq = batch, max_seq

    def pages(self) -> tuple[int, int]:
        """(free pages, pool pages) of a paged batch; (0, 0) otherwise."""
        f, t = C.c_size_t(0), C.c_size_t(0)
        check(lib.ifx_kv_batch_pages(self._h, C.byref(f), C.byref(t)), "kv_batch_pages")
        return int(f.value), int(t.value)

    def close(self):
        if getattr(self, "_h", None) is not None and self._h.value:
            lib.ifx_kv_batch_free(self._h)
            self._h = None

    def __del__(self):
        self.close()

    def len(self, seq: int) -> int:
        n = C.c_size_t(0)
        check(lib.ifx_kv_batch_len(self._h, seq, C.byref(n)), "kv_batch_len")
        return int(n.value)

    def prefill(self, seq: int, ids, last_row_only: bool = False) -> np.ndarray:
        m = self._model
        ids = np.ascontiguousarray(ids, np.uint32)
        rows = 1 if last_row_only else ids.size
        out = np.empty(rows * m.vocab, np.float32)
        check(lib.ifx_prefill_seq(m._h, self._h, seq, _u32(ids), ids.size, _f32(out),
                                  1 if last_row_only else 0), "prefill_seq")
        return out.reshape(rows, m.vocab)

    def decode_step(self, tokens, want_logits: bool = True):
        """One step of every sequence: (logits [batch, vocab] or None, argmax [batch])."""
        m = self._model
        t = np.ascontiguousarray(tokens, np.uint32)
        logits = np.empty(self.batch * m.vocab, np.float32) if want_logits else None
        amax = np.empty(self.batch, np.uint32)
        check(lib.ifx_decode_step_batch(m._h, self._h, _u32(t), _f32(logits) if want_logits else None,
                                        _u32(amax)), "decode_step_batch")
        return (logits.reshape(self.batch, m.vocab) if want_logits else None), amax

    def decode_step_seqs(self, seqs, tokens, want_logits: bool = True):
        """One step of the listed (distinct) sequences only; row i of the
        result (logits [n, vocab] or None, argmax [n]) belongs to seqs[i]."""
        m = self._model
        s = np.ascontiguousarray(seqs, np.int32)
        t = np.ascontiguousarray(tokens, np.uint32)
        if s.size != t.size:
            raise ValueError("one token per listed sequence")
        logits = np.empty(max(1, s.size) * m.vocab, np.float32) if want_logits else None
        amax = np.empty(max(1, s.size), np.uint32)
        check(lib.ifx_decode_step_batch_seqs(m._h, self._h, s.ctypes.data_as(C.POINTER(C.c_int)),
                                             int(s.size), _u32(t),
                                             _f32(logits) if want_logits else None, _u32(amax)),
              "decode_step_batch_seqs")
        return (logits[: s.size * m.vocab].reshape(s.size, m.vocab) if want_logits else None), amax[: s.size]

    def reset(self, seq: int) -> None:
        """KvCache::clear of one sequence, so a new request can take its place."""
        check(lib.ifx_kv_batch_reset(self._model._h, self._h, seq), "kv_batch_reset")

    def decode_greedy(self, tokens, n_steps: int, timed: bool = False):
        """n_steps greedy steps of every sequence: (tokens [n_steps, batch], device_ms)."""
        m = self._model
        t = np.ascontiguousarray(tokens, np.uint32)
        out = np.empty(max(n_steps, 1) * self.batch, np.uint32)
        ms = C.c_float(0.0)
        check(lib.ifx_decode_greedy_batch(m._h, self._h, _u32(t), n_steps, _u32(out),
                                          C.byref(ms) if timed else None), "decode_greedy_batch")
        return out[: n_steps * self.batch].reshape(n_steps, self.batch), (float(ms.value) if timed else None)


@dataclass
class Sampler:
    """Sampler (src/sampler.rs:8-16); sampling runs on the device."""

    temperature: float = 0.0
    top_k: int = 0
    top_p: float = 1.0

    @classmethod
    def greedy(cls) -> "Sampler":
        return cls(0.0, 0, 1.0)

    def _c(self) -> SamplerC:
        return SamplerC(self.temperature, self.top_k, self.top_p)

    def sample(self, model: Model, seed: int = 0, offset: int = 0) -> int:
        """Sample from the model's latest logits (prefill or decode_step)."""
        out = C.c_uint32()
        s = self._c()
        check(lib.ifx_sample(model._h, C.byref(s), seed, offset, C.byref(out)), "Sampler::sample")
        return int(out.value)


__all__ = ["Model", "KvCache", "KvBatch", "Sampler", "IfxError", "load_opts"]
