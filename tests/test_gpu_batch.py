"""Batched decode (B independent sequences per step) against the CPU oracle.

Each sequence is prefilled with its own prompt (different lengths, so the
sequences sit at different positions), then all of them step together
through the small-batch GEMM and the batched split-K attention. Every
sequence's logits must match the oracle's single-sequence decode at the
north star's bar (|gpu - ref| <= 2e-2 + 1e-2 |ref|), the batched argmax must
be the argmax of those logits, and the device-fed greedy loop must produce
the same tokens as stepping one token at a time.
"""
import os

import numpy as np
import pytest

from inferox_b200 import IfxError, Model, synth
from oracle import refcpu as R

pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-2, 1e-2
R.set_threads(os.cpu_count() or 8)


def _close(g, r):
    return np.all(np.abs(g - r) <= ATOL + RTOL * np.abs(r))


def _model(name):
    if name == "1b":
        return synth.build("1b")
    if name in ("grp6", "grp8"):  # 6 / 8 query heads per kv head (the 70B shape has 8)
        heads = 12 if name == "grp6" else 16
        return synth.build(None, vocab=2048, dim=64 * heads, n_layers=2, n_heads=heads, n_kv_heads=2,
                           ffn=1024, context=128, rope_base=10000.0, mix=1, seed=33)
    mix = 1 if name == "small_q4km" else 0  # Q4_K_M mix, or all Q8_0
    return synth.build(None, vocab=2048, dim=512, n_layers=2, n_heads=8, n_kv_heads=2, ffn=1024,
                       context=128, rope_base=500000.0, mix=mix, seed=31)


@pytest.mark.parametrize("name,batch,steps", [("small_q4km", 5, 4), ("small_q8", 3, 3), ("1b", 3, 2),
                                              ("grp6", 3, 3), ("grp8", 4, 3)])
def test_batched_decode_matches_oracle(name, batch, steps):
    g = _model(name)
    m, o = Model.from_bytes(g), R.Model(g)
    V, L = int(m.config.vocab_size), int(m.config.n_layers)
    kb = m.kv_batch(batch, 96)
    prompts = [synth.prompt_ids(V, 4 + 3 * b, seed=10 + b) for b in range(batch)]
    okv = [o.kv_cache(L, 96) for _ in range(batch)]
    toks = []
    for b in range(batch):
        gl = kb.prefill(b, prompts[b], True)[0]
        rl = o.prefill(prompts[b], okv[b], True)[0]
        assert _close(gl, rl), (b, float(np.max(np.abs(gl - rl))))
        toks.append(R.argmax(rl))
    for step in range(steps):
        logits, amax = kb.decode_step(toks)
        for b in range(batch):
            rl = o.decode_step(toks[b], okv[b])
            assert _close(logits[b], rl), (step, b, float(np.max(np.abs(logits[b] - rl))))
            assert int(amax[b]) == R.argmax(logits[b])
            toks[b] = R.argmax(rl)
    assert [kb.len(b) for b in range(batch)] == [len(p) + steps for p in prompts]


def test_batched_greedy_loop_equals_stepping():
    g = _model("small_q4km")
    m = Model.from_bytes(g)
    V = int(m.config.vocab_size)
    prompts = [synth.prompt_ids(V, 5 + 2 * b, seed=40 + b) for b in range(4)]
    a, b_ = m.kv_batch(4, 64), m.kv_batch(4, 64)
    first = []
    for s, p in enumerate(prompts):
        first.append(int(np.argmax(a.prefill(s, p, True)[0])))
        b_.prefill(s, p, True)
    toks, ms = a.decode_greedy(first, 6, timed=True)
    assert ms is not None and ms > 0
    cur = list(first)
    for i in range(6):
        _, amax = b_.decode_step(cur, want_logits=False)
        assert np.array_equal(amax, toks[i]), i
        cur = [int(t) for t in amax]


def test_batched_decode_errors():
    m = Model.from_bytes(_model("small_q8"))
    kb = m.kv_batch(2, 8)
    kb.prefill(0, [5, 6, 7], True)
    kb.prefill(1, [8], True)
    with pytest.raises(IfxError) as e:
        kb.decode_step([5, int(m.config.vocab_size)])  # forward.rs:552-554
    assert e.value.name == "InvalidTensorIndex"
    with pytest.raises(IfxError):
        kb.prefill(2, [1])  # no such sequence
    with pytest.raises(IfxError):
        m.kv_batch(33, 8)  # at most 32 sequences
    kb.decode_greedy([1, 2], 5)  # sequence 0 reaches the 8-row capacity
    with pytest.raises(IfxError) as e:
        kb.decode_step([1, 2])
    assert e.value.name == "InvalidTensorIndex"


def test_subset_steps_and_slot_reuse():
    """Continuous batching: steps over changing subsets of the sequences, and a
    slot reset and refilled by a new request, each sequence against the
    oracle's single-sequence decode."""
    g = _model("small_q4km")
    m, o = Model.from_bytes(g), R.Model(g)
    V, L = int(m.config.vocab_size), int(m.config.n_layers)
    kb = m.kv_batch(4, 64)
    okv, toks = {}, {}
    for s in (0, 2, 3):  # slot 1 starts empty
        p = synth.prompt_ids(V, 5 + s, seed=60 + s)
        okv[s] = o.kv_cache(L, 64)
        kb.prefill(s, p, True)
        toks[s] = R.argmax(o.prefill(p, okv[s], True)[0])

    def step(seqs):
        logits, amax = kb.decode_step_seqs(seqs, [toks[s] for s in seqs])
        for i, s in enumerate(seqs):
            rl = o.decode_step(toks[s], okv[s])
            assert _close(logits[i], rl), (seqs, s, float(np.max(np.abs(logits[i] - rl))))
            assert int(amax[i]) == R.argmax(logits[i])
            toks[s] = R.argmax(rl)

    for seqs in ([2, 0], [3], [0, 3, 2], [2, 0]):
        step(seqs)
    assert [kb.len(s) for s in range(4)] == [5 + 3, 0, 7 + 3, 8 + 2]
    kb.reset(0)  # a finished request leaves; a new one takes its slot
    assert kb.len(0) == 0
    p = synth.prompt_ids(V, 6, seed=99)
    okv[0] = o.kv_cache(L, 64)
    kb.prefill(0, p, True)
    toks[0] = R.argmax(o.prefill(p, okv[0], True)[0])
    okv[1], toks[1] = o.kv_cache(L, 64), 5  # slot 1 decodes from an empty cache
    step([1, 0])
    step([3, 1, 2, 0])
    logits, _ = kb.decode_step([toks[s] for s in range(4)])  # the whole batch again
    for s in range(4):
        assert _close(logits[s], o.decode_step(toks[s], okv[s]))
    for bad in ([1, 1], [4], []):
        with pytest.raises(IfxError):
            kb.decode_step_seqs(bad, [3] * len(bad))
    with pytest.raises(IfxError):
        kb.reset(4)


@pytest.mark.parametrize("name", ["grp6", "grp8"])
def test_single_sequence_decode_wide_groups(name):
    """The persistent kernel's tensor-core attention with two 8-column tiles
    (five to eight query heads per kv head) against the oracle, past one
    split of cached rows."""
    g = _model(name)
    m, o = Model.from_bytes(g), R.Model(g)
    V, L = int(m.config.vocab_size), int(m.config.n_layers)
    kv, okv = m.kv_cache(128), o.kv_cache(L, 128)
    p = synth.prompt_ids(V, 90, seed=5)
    gl, rl = m.prefill(p, kv, True)[0], o.prefill(p, okv, True)[0]
    assert _close(gl, rl)
    tok = R.argmax(rl)
    for i in range(6):
        gl, rl = m.decode_step(tok, kv), o.decode_step(tok, okv)
        assert _close(gl, rl), (i, float(np.max(np.abs(gl - rl))))
        tok = R.argmax(rl)
    assert kv.decode_kernels() == 1


@pytest.mark.parametrize("paged", [False, True])
def test_wide_batch_long_context(paged):
    """16 sequences x 8 kv heads (128 pairs, as in the 8B batch-16 step) at
    contexts of 300-700 positions: the attention runs one 8-warp CTA per
    (sequence, kv head) streaming its whole context with no split combine.
    Every sequence's logits against the oracle's single-sequence decode."""
    g = synth.build(None, vocab=1024, dim=1024, n_layers=2, n_heads=16, n_kv_heads=8, ffn=1024,
                    context=1024, rope_base=500000.0, mix=1, seed=71)
    m, o = Model.from_bytes(g), R.Model(g)
    V, L = int(m.config.vocab_size), int(m.config.n_layers)
    B, max_seq = 16, 768
    kb = m.kv_batch(B, max_seq, pages=B * 12 if paged else 0)
    prompts = [synth.prompt_ids(V, 300 + 25 * b, seed=90 + b) for b in range(B)]
    okv = [o.kv_cache(L, max_seq) for _ in range(B)]
    toks = []
    for b in range(B):
        kb.prefill(b, prompts[b], True)
        toks.append(R.argmax(o.prefill(prompts[b], okv[b], True)[0]))
    for step in range(2):
        logits, _ = kb.decode_step(toks)
        for b in range(B):
            rl = o.decode_step(toks[b], okv[b])
            assert _close(logits[b], rl), (step, b, float(np.max(np.abs(logits[b] - rl))))
            toks[b] = R.argmax(rl)
