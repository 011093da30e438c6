"""Tensor parallelism over the C ABI: communicators and weight shards.

    uid = tp.unique_id()                     # on rank 0; send the bytes to every rank
    comm = tp.Comm(uid, world, rank, device)  # collective
    model = Model.from_bytes(g, device=device, tp_size=world, tp_rank=rank,
                             nccl_comm=comm.handle)

The split (Megatron): Wq/Wk/Wv, W1/W3 and the vocab projection by rows, Wo
and W2 by their input dimension, the KV cache by kv head.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from ._lib import check, lib


def unique_id() -> bytes:
    buf = (C.c_char * 128)()
    check(lib.ifx_tp_unique_id(buf), "tp_unique_id")
    return bytes(buf)


class Comm:
    """An NCCL communicator made by the library's own NCCL instance."""

    def __init__(self, uid: bytes, nranks: int, rank: int, device: int):
        assert len(uid) == 128
        h = C.c_void_p()
        idb = (C.c_char * 128).from_buffer_copy(uid)
        check(lib.ifx_tp_comm_create(idb, nranks, rank, device, C.byref(h)), "tp_comm_create")
        self.handle = h.value

    def close(self):
        if getattr(self, "handle", None):
            lib.ifx_tp_comm_destroy(C.c_void_p(self.handle))
            self.handle = None


def shard(ttype: int, gguf_bytes, rows: int, cols: int, split_k: bool, tp: int,
          rank: int) -> bytes:
    """The bytes of the shard `rank` of `tp` holds (host only)."""
    src = np.frombuffer(bytes(gguf_bytes), np.uint8)
    n = C.c_size_t()
    check(lib.ifx_tp_shard(ttype, src.ctypes.data_as(C.c_void_p), src.nbytes, rows, cols,
                           1 if split_k else 0, tp, rank, None, C.byref(n)), "tp_shard")
    out = np.empty(n.value, np.uint8)
    check(lib.ifx_tp_shard(ttype, src.ctypes.data_as(C.c_void_p), src.nbytes, rows, cols,
                           1 if split_k else 0, tp, rank, out.ctypes.data_as(C.c_void_p),
                           C.byref(n)), "tp_shard")
    return out.tobytes()
