"""Tensor-parallel decode and prefill on 2, 4 and 8 GPUs against the CPU oracle.

Spawned ranks, each on its own GPU, load the same synthetic GGUF with
tp_size equal to the rank count through a communicator made by the library (ifx_tp_unique_id /
ifx_tp_comm_create), run a prefill and greedy decode steps, and hand their
(all-gathered, hence full) logits to the parent, which holds them to the
oracle at the parity bar and to each other bit for bit. Decode runs both
ways: the persistent kernel with its all-reduces over peer memory inside
the step, and the per-op kernels with NCCL between them. The ranks do no
checking themselves, so none can leave another waiting in a
collective; the parent kills them all if they do not report in time. NVLS is
off (NCCL_NVLS_ENABLE=0) and the kernel's own waits use plain peer loads.
Each case is skipped when the box has fewer GPUs than it has ranks.
"""
import os

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from inferox_b200 import synth, tp
from oracle import refcpu as R

pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-2, 1e-2
R.set_threads(os.cpu_count() or 8)


def _rank(rank, world, uid, g, prompt, steps, q, persistent):
    try:
        os.environ["NCCL_NVLS_ENABLE"] = "0"
        from inferox_b200 import Model
        comm = tp.Comm(uid, world, rank, rank)
        m = Model.from_bytes(g, device=rank, tp_size=world, tp_rank=rank, nccl_comm=comm.handle,
                             persistent_decode=persistent)
        kv = m.kv_cache(128)
        out = {"prefill_last": m.prefill(prompt, kv, True)[0]}
        out["prefill_all"] = m.prefill(prompt, m.kv_cache(128), False)
        logs = []
        for t in steps:
            logs.append(m.decode_step(int(t), kv))
        out["decode"] = np.stack(logs)
        toks, _ = m.decode_greedy(int(steps[-1]), 6, kv)
        out["greedy"] = toks
        out["kernels"] = kv.decode_kernels()
        del kv, m
        comm.close()
        q.put((rank, out))
    except Exception as e:
        q.put((rank, repr(e)))


def _close(a, b):
    return np.all(np.abs(a - b) <= ATOL + RTOL * np.abs(b))


def _run(world, mix, persistent, heads, kv_heads):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    # each rank's slice of the FFN rows (W2's columns) is a whole 256-column super-block
    g = synth.build(None, vocab=2048, dim=64 * heads, n_layers=2, n_heads=heads,
                    n_kv_heads=kv_heads, ffn=max(1024, 256 * world), context=128,
                    rope_base=500000.0, mix=mix, seed=21)
    prompt = synth.prompt_ids(2048, 10, seed=3)
    o = R.Model(g)
    okv = o.kv_cache(2, 128)
    ref_last = o.prefill(prompt, okv, True)[0]
    ref_all = o.prefill(prompt, o.kv_cache(2, 128), False)
    steps = [int(R.argmax(ref_last))]
    ref_dec = []
    for _ in range(4):
        r = o.decode_step(steps[-1], okv)
        ref_dec.append(r)
        steps.append(int(R.argmax(r)))
    steps = steps[:4]
    uid = tp.unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, world, uid, g, prompt, steps, q, persistent))
             for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in procs:
            r, out = q.get(timeout=240)
            res[r] = out
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    for r in range(world):
        assert isinstance(res.get(r), dict), res.get(r)
    a = res[0]
    for r in range(1, world):  # gathered logits are the same on every rank
        for k in ("prefill_last", "prefill_all", "decode"):
            assert np.array_equal(a[k], res[r][k]), (r, k)
        assert np.array_equal(a["greedy"], res[r]["greedy"]), r
    assert _close(a["prefill_last"], ref_last), float(np.max(np.abs(a["prefill_last"] - ref_last)))
    assert _close(a["prefill_all"], ref_all), float(np.max(np.abs(a["prefill_all"] - ref_all)))
    for i, r in enumerate(ref_dec):
        assert _close(a["decode"][i], r), (i, float(np.max(np.abs(a["decode"][i] - r))))
    # the persistent kernel, or the per-op kernels with the collectives between them
    assert a["kernels"] == (1 if persistent else 3 + 5 * 2)


@pytest.mark.parametrize("mix,persistent,heads", [(1, True, 8), (0, True, 8), (1, False, 8),
                                                  (0, False, 8), (1, True, 16)])
def test_tp2_matches_oracle(mix, persistent, heads):
    """mix 1: Q4_K_M, 0: all Q8_0; heads 16 over 2 kv heads: 8 query heads
    per kv head on each rank, as in the 70B shape."""
    _run(2, mix, persistent, heads, 2)


@pytest.mark.parametrize("world,persistent,heads", [(4, True, 16), (4, False, 16), (8, True, 32),
                                                    (8, False, 32)])
def test_tp4_tp8_match_oracle(world, persistent, heads):
    """Four and eight ranks, one kv head each (the 8B shape's split at tp8,
    the 70B shape's at tp8 with 32 query heads: 4 per kv head), Q4_K_M."""
    _run(world, 1, persistent, heads, world)
