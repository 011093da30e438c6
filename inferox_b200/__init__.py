"""inferox_b200 — sm_100a implementation of phraakture/inferox's token loop.

The compute lives in libinferox_b200.so (CUDA kernels + C ABI, see
include/inferox.h); this package is the host-side mirror of the reference's
Rust API. Import fails loudly if the library is missing: there is no CPU
fallback.
"""
from ._lib import IfxError, header_symbols, lib  # noqa: F401
from .model import KvBatch, KvCache, Model, Sampler, load_opts  # noqa: F401
from .tokenizer import BpeTokenizer  # noqa: F401

__all__ = ["Model", "KvCache", "KvBatch", "Sampler", "BpeTokenizer", "IfxError", "load_opts", "lib",
           "header_symbols"]
