"""Tensor-parallel partition math and collective protocol on CPU: two gloo
ranks (world_size 2, 127.0.0.1).

Each rank takes its shard of a quantised weight through the library's
ifx_tp_shard, dequantises it with the oracle (exact) and computes its part
of y = W x:
  * a row split (Wq/Wk/Wv, W1/W3, vocab) gives a slice of y: all_gather;
  * an input-dimension split (Wo, W2) gives a partial sum: all_reduce.
Either way the result must equal the oracle's full product. The vocab
argmax protocol is checked the same way: each rank's 64-bit key (ordered
value bits << 32 | global index), then a MAX all-reduce, must give the
reference argmax including its last-index-on-ties rule.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from inferox_b200 import synth, tp
from oracle import refcpu as R

TYPES = [(12, 256), (14, 256), (7, 32), (2, 32)]  # Q4_K, Q6_K, Q8_0, Q4_0 (block elems)


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def ordered_bits(v: np.float32) -> int:
    """The key order of the device argmax: monotone in the float value."""
    b = int(np.float32(v).view(np.uint32))
    return (b | 0x80000000) if b < 0x80000000 else (~b) & 0xFFFFFFFF


def _worker(rank: int, world: int, port: int, q: "mp.Queue"):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world)
        rng = np.random.default_rng(7)
        for ttype, be in TYPES:
            rows, cols = 64, 4 * be * world
            w = rng.standard_normal(rows * cols).astype(np.float32) * 0.02
            qb = synth.quantize(ttype, w)
            x = rng.standard_normal(cols)
            full = R.dequantize(ttype, qb, rows * cols).reshape(rows, cols).astype(np.float64) @ x
            # row split: a slice of y per rank
            sh = tp.shard(ttype, qb, rows, cols, False, world, rank)
            part = R.dequantize(ttype, sh, rows // world * cols).reshape(rows // world, cols)
            y_loc = torch.from_numpy(part.astype(np.float64) @ x)
            got = [torch.empty_like(y_loc) for _ in range(world)]
            dist.all_gather(got, y_loc)
            assert np.allclose(torch.cat(got).numpy(), full, rtol=1e-12, atol=1e-12), ttype
            # input-dimension split: a partial sum per rank
            sh = tp.shard(ttype, qb, rows, cols, True, world, rank)
            kc = cols // world
            part = R.dequantize(ttype, sh, rows * kc).reshape(rows, kc)
            y_part = torch.from_numpy(part.astype(np.float64) @ x[rank * kc:(rank + 1) * kc])
            dist.all_reduce(y_part)
            assert np.allclose(y_part.numpy(), full, rtol=1e-10, atol=1e-12), ttype
        # vocab-sharded argmax with a tie that spans both shards
        V = 1000
        logits = rng.standard_normal(V).astype(np.float32)
        logits[[123, 987]] = np.float32(5.0)  # the reference keeps the last index
        vl = V // world
        mine = logits[rank * vl:(rank + 1) * vl]
        keys = [(ordered_bits(v) << 32) | (rank * vl + i) for i, v in enumerate(mine)]
        # the device reduces unsigned 64-bit keys (ncclUint64 max); gloo has
        # signed int64 only, so shift by 2^63 (order preserving)
        k = torch.tensor([max(keys) - (1 << 63)], dtype=torch.int64)
        dist.all_reduce(k, op=dist.ReduceOp.MAX)
        tok = (int(k.item()) + (1 << 63)) & 0xFFFFFFFF
        assert tok == R.argmax(logits) == 987, tok
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, "ok"))
    except Exception as e:  # report to the parent instead of hanging it
        q.put((rank, repr(e)))


def test_tp_partitions_on_two_gloo_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert res == {0: "ok", 1: "ok"}, res


@pytest.mark.parametrize("ttype,be", TYPES)
def test_tp_shard_rejects_ragged_splits(ttype, be):
    w = np.zeros(8 * be * 3, np.float32)
    qb = synth.quantize(ttype, w)
    from inferox_b200 import IfxError
    with pytest.raises(IfxError) as e:  # 3 blocks per row do not split in two
        tp.shard(ttype, qb, 8, be * 3, True, 2, 0)
    assert e.value.name == "Shape"
    with pytest.raises(IfxError):  # 8 rows do not split in three
        tp.shard(ttype, qb, 8, be * 3, False, 3, 0)
