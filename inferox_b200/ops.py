"""Mirror of src/ops.rs (and the dequantiser, src/gguf/dequant.rs) over the
op-level C ABI. Arguments are CUDA tensors (torch is used only to hold device
memory and streams); every call runs the library's sm_100a kernels.

Shape mismatches raise IfxError("Shape") where the reference panics.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import torch

from ._lib import IfxError, SamplerC, check, lib


def _p(t: torch.Tensor) -> C.c_void_p:
    if not t.is_cuda:
        raise IfxError(24, "expected a CUDA tensor")
    if not t.is_contiguous():
        raise IfxError(24, "expected a contiguous tensor")
    return C.c_void_p(t.data_ptr())


def _s() -> C.c_void_p:
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


def _need(cond: bool, what: str):
    if not cond:
        raise IfxError(20, what)


def dequantize(ttype: int, data: torch.Tensor, n_out: int) -> torch.Tensor:
    """dequantize_f32 (dequant.rs:10-31): uint8 CUDA bytes -> f32 [n_out]."""
    out = torch.empty(n_out, dtype=torch.float32, device=data.device)
    check(lib.ifx_op_dequantize(ttype, _p(data), data.numel(), _p(out), n_out, _s()), "dequantize")
    return out


def matmul(a, b, m, n, k) -> torch.Tensor:  # ops.rs:15-26
    _need(a.numel() == m * k and b.numel() == k * n, "matmul shape mismatch")
    c = torch.empty(m * n, dtype=torch.float32, device=a.device)
    check(lib.ifx_op_matmul(_p(a), _p(b), _p(c), m, n, k, _s()), "matmul")
    return c


def matmul_t(a, b, m, n, k) -> torch.Tensor:  # ops.rs:33-44
    _need(a.numel() == m * k and b.numel() == n * k, "matmul_t shape mismatch")
    c = torch.empty(m * n, dtype=torch.float32, device=a.device)
    check(lib.ifx_op_matmul_t(_p(a), _p(b), _p(c), m, n, k, _s()), "matmul_t")
    return c


class QMatrix:
    """A quantised [rows, cols] weight uploaded and repacked once."""

    def __init__(self, ttype: int, gguf_bytes: bytes | np.ndarray, rows: int, cols: int,
                 device: int = 0):
        buf = np.frombuffer(bytes(gguf_bytes), np.uint8) if not isinstance(gguf_bytes, np.ndarray) \
            else np.ascontiguousarray(gguf_bytes, np.uint8)
        h = C.c_void_p()
        check(lib.ifx_qmatrix_create(ttype, buf.ctypes.data_as(C.c_void_p), buf.nbytes, rows, cols,
                                     device, C.byref(h)), "qmatrix_create")
        self._h = h
        self.rows, self.cols, self.type = rows, cols, ttype

    def __del__(self):
        if getattr(self, "_h", None) is not None and self._h.value:
            lib.ifx_qmatrix_free(self._h)
            self._h = None


def matmul_t_q(a: torch.Tensor, w: QMatrix, m: int) -> torch.Tensor:
    """C[m, rows] = A[m, cols] W^T with the fused dequant kernels."""
    _need(a.numel() == m * w.cols, "matmul_t_q shape mismatch")
    c = torch.empty(m * w.rows, dtype=torch.float32, device=a.device)
    check(lib.ifx_op_matmul_t_q(_p(a), w._h, _p(c), m, _s()), "matmul_t_q")
    return c


def bench_matmul_t_q(a: torch.Tensor, w: QMatrix, m: int, reps: int = 10) -> float:
    """ms per call of the fused dequant matmul the token loop runs at batch m
    (GEMV at 1, small-batch GEMM up to 32, prefill GEMM above), each launch
    timed alone with the weights coming from HBM."""
    _need(a.numel() == m * w.cols, "bench_matmul_t_q shape mismatch")
    c = torch.empty(m * w.rows, dtype=torch.float32, device=a.device)
    ms = C.c_float(0.0)
    check(lib.ifx_bench_matmul_t_q(_p(a), w._h, _p(c), m, reps, C.byref(ms)), "bench_matmul_t_q")
    return float(ms.value)


def rms_norm(x, w, eps):  # ops.rs:155-168 (in place)
    _need(x.numel() == w.numel(), "RMSNorm weight length mismatch")
    check(lib.ifx_op_rms_norm_rows(_p(x), _p(w), eps, 1, w.numel(), _s()), "rms_norm")
    return x


def rms_norm_rows(x, w, eps, rows):  # ops.rs:173-180 (in place)
    _need(x.numel() == rows * w.numel(), "RMSNorm rows shape mismatch")
    check(lib.ifx_op_rms_norm_rows(_p(x), _p(w), eps, rows, w.numel(), _s()), "rms_norm_rows")
    return x


def silu(x):  # ops.rs:183-187 (in place)
    check(lib.ifx_op_silu(_p(x), x.numel(), _s()), "silu")
    return x


def swiglu(gate, up):  # ops.rs:190-197
    _need(gate.numel() == up.numel(), "SwiGLU gate/up length mismatch")
    out = torch.empty_like(gate)
    check(lib.ifx_op_swiglu(_p(gate), _p(up), _p(out), gate.numel(), _s()), "swiglu")
    return out


def add_in_place(out, b):  # ops.rs:212-217
    _need(out.numel() == b.numel(), "add length mismatch")
    check(lib.ifx_op_add_in_place(_p(out), _p(b), out.numel(), _s()), "add_in_place")
    return out


def softmax_rows(x, rows, cols):  # ops.rs:223-239 (in place)
    _need(x.numel() == rows * cols, "softmax shape mismatch")
    check(lib.ifx_op_softmax_rows(_p(x), rows, cols, _s()), "softmax_rows")
    return x


def embedding_lookup(emb, ids, hidden):  # ops.rs:246-258
    out = torch.empty(ids.numel() * hidden, dtype=torch.float32, device=emb.device)
    check(lib.ifx_op_embedding_lookup(_p(emb), emb.numel(), _p(ids), ids.numel(), hidden, _p(out),
                                      _s()), "embedding_lookup")
    return out


def rope(x, seq_len, n_heads, head_dim, rope_dim, base, pos0=0):  # ops.rs:265-287
    _need(x.numel() == seq_len * n_heads * head_dim, "rope shape mismatch")
    check(lib.ifx_op_rope(_p(x), seq_len, n_heads, head_dim, rope_dim, base, pos0, _s()), "rope")
    return x


def argmax(x) -> int:  # forward.rs:615-622
    out = torch.zeros(1, dtype=torch.int32, device=x.device)
    check(lib.ifx_op_argmax(_p(x), x.numel(), _p(out), _s()), "argmax")
    return int(out.item())


def sample_u(logits, temperature, top_k, top_p, u) -> int:
    """Sampler::sample (sampler.rs:28-73) with the uniform draw supplied."""
    s = SamplerC(temperature, top_k, top_p)
    tok = C.c_uint32()
    check(lib.ifx_op_sample_u(_p(logits), logits.numel(), C.byref(s), float(u), C.byref(tok),
                              _s()), "sample_u")
    return int(tok.value)
