"""ctypes binding of include/inferox.h (the C ABI of libinferox_b200.so).

The library is the product: there is no CPU fallback. If the shared object is
missing or fails to load, importing this module raises immediately.
"""
from __future__ import annotations

import ctypes as C
import os
import re

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libinferox_b200.so")
HEADER = os.path.join(os.path.dirname(HERE), "include", "inferox.h")

STATUS = {
    0: "Ok", 1: "Io", 2: "InvalidMagic", 3: "UnsupportedVersion", 4: "UnknownValueType",
    5: "UnknownTensorType", 6: "InvalidUtf8", 7: "InvalidShape", 8: "UnexpectedEof",
    9: "TensorNotFound", 10: "InvalidTensorIndex", 11: "TensorOffsetOverflow",
    12: "UnsupportedArchitecture", 20: "Shape", 21: "Cuda", 22: "Nccl", 23: "Timeout",
    24: "InvalidArgument", 25: "OutOfMemory", 26: "Unsupported", 27: "Json",
    28: "UnsupportedModel",
}

TYPE_F32, TYPE_F16, TYPE_Q4_0, TYPE_Q8_0, TYPE_Q4_K, TYPE_Q6_K, TYPE_Q8_K = 0, 1, 2, 7, 12, 14, 15


class IfxError(RuntimeError):
    """A non-zero ifx_status; `.name` mirrors the gguf::Error variant."""

    def __init__(self, code: int, message: str):
        self.code = code
        self.name = STATUS.get(code, f"status{code}")
        super().__init__(f"{self.name}: {message}")


class Config(C.Structure):
    _fields_ = [
        ("vocab_size", C.c_uint32),
        ("hidden_size", C.c_uint64), ("n_layers", C.c_uint64), ("n_heads", C.c_uint64),
        ("n_kv_heads", C.c_uint64), ("head_dim", C.c_uint64),
        ("intermediate_size", C.c_uint64),
        ("norm_eps", C.c_float), ("rope_base", C.c_float),
        ("rope_dim", C.c_uint64), ("context_length", C.c_uint64),
        ("architecture", C.c_char * 64),
    ]


class LoadOpts(C.Structure):
    _fields_ = [
        ("device", C.c_int), ("tp_size", C.c_int), ("tp_rank", C.c_int),
        ("nccl_comm", C.c_void_p), ("rope_compat", C.c_int), ("use_graphs", C.c_int),
        ("persistent_decode", C.c_int), ("kquant_layout", C.c_int), ("tp_timeout_ms", C.c_int),
    ]


class SamplerC(C.Structure):
    _fields_ = [("temperature", C.c_float), ("top_k", C.c_uint64), ("top_p", C.c_float)]


class SynthSpec(C.Structure):
    _fields_ = [
        ("vocab", C.c_uint32), ("dim", C.c_uint32), ("n_layers", C.c_uint32),
        ("n_heads", C.c_uint32), ("n_kv_heads", C.c_uint32), ("ffn", C.c_uint32),
        ("context", C.c_uint32),
        ("rope_base", C.c_float), ("norm_eps", C.c_float), ("sigma", C.c_float),
        ("mix", C.c_int), ("tied", C.c_int), ("seed", C.c_uint64), ("threads", C.c_int),
    ]


def header_symbols() -> list[str]:
    """Every function the public header declares."""
    src = open(HEADER).read()
    return sorted(set(re.findall(r"\b(ifx_[a-z0-9_]+)\s*\(", src)))


def _load():
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"{LIB_PATH} is missing: build it with `python inferox_b200/build.py` "
            "(the CUDA library is the only implementation)")
    L = C.CDLL(LIB_PATH, mode=C.RTLD_GLOBAL)
    vp, sz, u32p, fp = C.c_void_p, C.c_size_t, C.POINTER(C.c_uint32), C.POINTER(C.c_float)
    st = C.c_int
    sig = {
        "ifx_last_error": (C.c_char_p, []),
        "ifx_status_name": (C.c_char_p, [st]),
        "ifx_version": (C.c_int, []),
        "ifx_load_opts_default": (None, [C.POINTER(LoadOpts)]),
        "ifx_model_load": (st, [C.c_char_p, C.POINTER(LoadOpts), C.POINTER(vp)]),
        "ifx_model_load_mem": (st, [vp, sz, C.POINTER(LoadOpts), C.POINTER(vp)]),
        "ifx_model_free": (None, [vp]),
        "ifx_model_config": (st, [vp, C.POINTER(Config)]),
        "ifx_model_decode_weight_bytes": (C.c_uint64, [vp]),
        "ifx_kv_create": (st, [vp, sz, C.POINTER(vp)]),
        "ifx_kv_free": (None, [vp]),
        "ifx_kv_clear": (st, [vp]),
        "ifx_kv_len": (sz, [vp]),
        "ifx_kv_decode_kernels": (C.c_int, [vp]),
        "ifx_tp_unique_id": (st, [vp]),
        "ifx_tp_comm_create": (st, [vp, C.c_int, C.c_int, C.c_int, C.POINTER(vp)]),
        "ifx_tp_comm_destroy": (None, [vp]),
        "ifx_tp_shard": (st, [C.c_int, vp, sz, sz, sz, C.c_int, C.c_int, C.c_int, vp, C.POINTER(sz)]),
        "ifx_kv_read": (st, [vp, sz, C.c_int, fp]),
        "ifx_prefill": (st, [vp, vp, u32p, sz, fp, C.c_int]),
        "ifx_decode_step": (st, [vp, vp, C.c_uint32, fp]),
        "ifx_forward": (st, [vp, u32p, sz, fp, C.c_int]),
        "ifx_generate": (st, [vp, vp, u32p, sz, sz, u32p]),
        "ifx_sample": (st, [vp, C.POINTER(SamplerC), C.c_uint64, C.c_uint64, u32p]),
        "ifx_decode_greedy": (st, [vp, vp, C.c_uint32, sz, u32p, fp]),
        "ifx_bench_kernel": (st, [vp, vp, C.c_char_p, C.c_int, fp, C.POINTER(C.c_uint64)]),
        "ifx_kv_batch_create": (st, [vp, sz, C.c_int, C.POINTER(vp)]),
        "ifx_kv_batch_create_paged": (st, [vp, sz, C.c_int, sz, C.POINTER(vp)]),
        "ifx_kv_batch_pages": (st, [vp, C.POINTER(sz), C.POINTER(sz)]),
        "ifx_kv_batch_free": (None, [vp]),
        "ifx_kv_batch_len": (st, [vp, C.c_int, C.POINTER(sz)]),
        "ifx_prefill_seq": (st, [vp, vp, C.c_int, u32p, sz, fp, C.c_int]),
        "ifx_decode_step_batch": (st, [vp, vp, u32p, fp, u32p]),
        "ifx_decode_step_batch_seqs": (st, [vp, vp, C.POINTER(C.c_int), C.c_int, u32p, fp, u32p]),
        "ifx_kv_batch_reset": (st, [vp, vp, C.c_int]),
        "ifx_decode_greedy_batch": (st, [vp, vp, u32p, sz, u32p, fp]),
        "ifx_op_dequantize": (st, [C.c_int, vp, sz, vp, sz, vp]),
        "ifx_op_matmul": (st, [vp, vp, vp, sz, sz, sz, vp]),
        "ifx_op_matmul_t": (st, [vp, vp, vp, sz, sz, sz, vp]),
        "ifx_qmatrix_create": (st, [C.c_int, vp, sz, sz, sz, C.c_int, C.POINTER(vp)]),
        "ifx_qmatrix_free": (None, [vp]),
        "ifx_op_matmul_t_q": (st, [vp, vp, vp, sz, vp]),
        "ifx_bench_matmul_t_q": (st, [vp, vp, vp, sz, C.c_int, fp]),
        "ifx_op_rms_norm_rows": (st, [vp, vp, C.c_float, sz, sz, vp]),
        "ifx_op_silu": (st, [vp, sz, vp]),
        "ifx_op_swiglu": (st, [vp, vp, vp, sz, vp]),
        "ifx_op_add_in_place": (st, [vp, vp, sz, vp]),
        "ifx_op_softmax_rows": (st, [vp, sz, sz, vp]),
        "ifx_op_embedding_lookup": (st, [vp, sz, vp, sz, sz, vp, vp]),
        "ifx_op_rope": (st, [vp, sz, sz, sz, sz, C.c_float, sz, vp]),
        "ifx_op_argmax": (st, [vp, sz, vp, vp]),
        "ifx_op_sample_u": (st, [vp, sz, C.POINTER(SamplerC), C.c_float, u32p, vp]),
        "ifx_op_sample_u_static": (st, [vp, sz, C.POINTER(SamplerC), C.c_float, vp, vp]),
        "ifx_kquant_from_ggml": (st, [C.c_uint32, vp, sz, vp, C.POINTER(C.c_int), C.POINTER(C.c_int)]),
        "ifx_tokenizer_load": (st, [C.c_char_p, C.POINTER(vp)]),
        "ifx_tokenizer_load_json": (st, [C.c_char_p, sz, C.POINTER(vp)]),
        "ifx_tokenizer_free": (None, [vp]),
        "ifx_tokenizer_encode": (st, [vp, C.c_char_p, sz, u32p, sz, C.POINTER(sz)]),
        "ifx_tokenizer_decode": (st, [vp, u32p, sz, C.c_char_p, sz, C.POINTER(sz)]),
        "ifx_tokenizer_vocab_size": (st, [vp, C.POINTER(sz)]),
        "ifx_synth_gguf": (st, [C.POINTER(SynthSpec), C.POINTER(vp), C.POINTER(sz)]),
        "ifx_synth_free": (None, [vp]),
        "ifx_quantize": (st, [C.c_int, vp, sz, vp]),
        "ifx_synth_normal": (st, [C.c_uint64, C.c_uint64, C.c_float, fp, sz]),
    }
    for name, (res, args) in sig.items():
        f = getattr(L, name)
        f.restype = res
        f.argtypes = args
    return L


lib = _load()


def check(code: int, what: str = "") -> None:
    if code != 0:
        msg = lib.ifx_last_error().decode(errors="replace")
        raise IfxError(code, f"{what}: {msg}" if what else msg)
