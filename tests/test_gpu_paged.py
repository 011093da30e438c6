"""Paged batch (sequences sharing a pool of 64-position cache pages) against
the CPU oracle.

The reference keeps one contiguous cache per sequence (src/model/cache.rs:7-13);
the paged batch gives the same results with the rows of every sequence in
pages taken from one pool. These tests prefill prompts that end on either
side of page boundaries, decode across a boundary (a page is taken in the
middle of decoding), run the pool dry (the step fails with OutOfMemory and no
length moves), and hand a reset sequence's pages, stale rows and all, to a
new request. Every sequence's logits are held to the oracle's single-sequence
decode at the north star's bar.
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


def _model():
    return synth.build(None, vocab=2048, dim=512, n_layers=2, n_heads=8, n_kv_heads=2, ffn=1024,
                       context=512, rope_base=500000.0, mix=1, seed=31)


def test_paged_decode_matches_oracle():
    g = _model()
    m, o = Model.from_bytes(g), R.Model(g)
    V, L = int(m.config.vocab_size), int(m.config.n_layers)
    lens = [60, 70, 130, 5]  # 1, 2, 3 and 1 pages; sequence 0 takes a page while decoding
    kb = m.kv_batch(len(lens), 256, pages=10)
    assert kb.pages() == (10, 10)
    okv, toks = [], []
    for s, n in enumerate(lens):
        p = synth.prompt_ids(V, n, seed=70 + s)
        okv.append(o.kv_cache(L, 256))
        gl = kb.prefill(s, p, True)[0]
        rl = o.prefill(p, okv[s], True)[0]
        assert _close(gl, rl), (s, float(np.max(np.abs(gl - rl))))
        toks.append(R.argmax(rl))
    assert kb.pages() == (10 - 7, 10)
    for step in range(8):
        logits, amax = kb.decode_step(toks)
        for s in range(len(lens)):
            rl = o.decode_step(toks[s], okv[s])
            assert _close(logits[s], rl), (step, s, float(np.max(np.abs(logits[s] - rl))))
            assert int(amax[s]) == R.argmax(logits[s])
            toks[s] = R.argmax(rl)
    assert [kb.len(s) for s in range(len(lens))] == [n + 8 for n in lens]
    assert kb.pages() == (10 - 8, 10)


def test_paged_greedy_loop_equals_stepping():
    g = _model()
    m = Model.from_bytes(g)
    V = int(m.config.vocab_size)
    prompts = [synth.prompt_ids(V, 58 + 3 * b, seed=40 + b) for b in range(3)]
    a, b_ = m.kv_batch(3, 128, pages=8), m.kv_batch(3, 128, pages=8)
    first = []
    for s, p in enumerate(prompts):
        first.append(int(np.argmax(a.prefill(s, p, True)[0])))
        b_.prefill(s, p, True)
    toks, _ = a.decode_greedy(first, 10)  # every sequence crosses position 64
    cur = list(first)
    for i in range(10):
        _, amax = b_.decode_step(cur, want_logits=False)
        assert np.array_equal(amax, toks[i]), i
        cur = [int(t) for t in amax]
    assert a.pages() == b_.pages() == (8 - 6, 8)


def test_pool_exhaustion_and_page_reuse():
    g = _model()
    m, o = Model.from_bytes(g), R.Model(g)
    V, L = int(m.config.vocab_size), int(m.config.n_layers)
    kb = m.kv_batch(2, 256, pages=3)
    p0 = synth.prompt_ids(V, 100, seed=1)
    o0 = o.kv_cache(L, 256)
    kb.prefill(0, p0, True)
    t0 = R.argmax(o.prefill(p0, o0, True)[0])
    assert kb.pages() == (1, 3)
    with pytest.raises(IfxError) as e:
        kb.prefill(1, synth.prompt_ids(V, 100, seed=2), True)  # needs 2 pages, 1 free
    assert e.value.name == "OutOfMemory"
    assert kb.len(1) == 0 and kb.pages() == (1, 3)
    p1 = synth.prompt_ids(V, 62, seed=3)
    o1 = o.kv_cache(L, 256)
    kb.prefill(1, p1, True)
    t1 = R.argmax(o.prefill(p1, o1, True)[0])
    assert kb.pages() == (0, 3)
    for _ in range(2):  # positions 62 and 63: still in sequence 1's first page
        logits, _ = kb.decode_step([t0, t1])
        for lg, (t, okv) in zip(logits, ((t0, o0), (t1, o1))):
            assert _close(lg, o.decode_step(t, okv))
        t0, t1 = R.argmax(logits[0]), R.argmax(logits[1])
    # position 64 of sequence 1 needs a page the pool no longer has
    with pytest.raises(IfxError) as e:
        kb.decode_step([t0, t1])
    assert e.value.name == "OutOfMemory"
    assert (kb.len(0), kb.len(1)) == (102, 64)
    kb.reset(0)  # a finished request returns its two pages
    assert kb.pages() == (2, 3) and kb.len(0) == 0
    logits, _ = kb.decode_step_seqs([1], [t1])  # now sequence 1 gets a page
    assert kb.len(1) == 65 and kb.pages() == (1, 3)
    assert _close(logits[0], o.decode_step(t1, o1))
    # a new request on the reset slot reuses a page that still holds old rows
    p2 = synth.prompt_ids(V, 40, seed=4)
    o2 = o.kv_cache(L, 256)
    gl = kb.prefill(0, p2, True)[0]
    rl = o.prefill(p2, o2, True)[0]
    assert _close(gl, rl)
    t2 = R.argmax(rl)
    logits, _ = kb.decode_step_seqs([0], [t2])
    rl = o.decode_step(t2, o2)
    assert _close(logits[0], rl), float(np.max(np.abs(logits[0] - rl)))


def test_paged_errors():
    m = Model.from_bytes(_model())
    with pytest.raises(IfxError):
        m.kv_batch(2, 64 * 64 + 1, pages=4)  # at most 64 pages of 64 rows per sequence
    kb = m.kv_batch(2, 64)
    assert kb.pages() == (0, 0)  # not a paged batch
