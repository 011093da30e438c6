"""The continuous-batching serving loop (inferox_b200.serving.Server) on the
GPU, end to end: requests of different prompt lengths and token budgets
arrive while others run, over a contiguous batch and over a paged pool small
enough that requests wait for pages or are preempted. Each request must be
a greedy decode of the reference model (src/model/forward.rs:592-622): the
oracle, teacher-forced with the request's own tokens, must find every
chosen token's logit within the parity tolerance of its maximum (two
implementations may break a near tie differently; everything else must
agree), and the first token of every request must be the oracle's argmax.
"""
import os

import numpy as np
import pytest

from inferox_b200 import Model, synth
from inferox_b200.serving import Server
from oracle import refcpu as R

pytestmark = pytest.mark.gpu

R.set_threads(os.cpu_count() or 8)


def _model():
    return synth.build(None, vocab=2048, dim=512, n_layers=2, n_heads=8, n_kv_heads=2, ffn=1024,
                       context=256, rope_base=500000.0, mix=1, seed=61)


def _check_greedy(o, prompt, tokens):
    """Teacher-forced: each token is a maximum of the oracle's logits within
    |d| <= 2e-2 + 1e-2 |max|; returns how many are the exact argmax."""
    kv = o.kv_cache(2, len(prompt) + len(tokens) + 1)
    logits = o.prefill(prompt, kv, True)[0]
    exact = 0
    for i, t in enumerate(tokens):
        mx = float(np.max(logits))
        assert logits[t] >= mx - (2e-2 + 1e-2 * abs(mx)), (i, t, float(logits[t]), mx)
        exact += int(t == R.argmax(logits))
        if i == 0:
            assert t == R.argmax(logits)
        if i + 1 < len(tokens):
            logits = o.decode_step(t, kv)
    return exact


@pytest.mark.parametrize("pages", [0, 5])  # contiguous slots; a 5-page (320-row) pool
def test_server_requests_match_solo_generate(pages):
    g = _model()
    m, o = Model.from_bytes(g), R.Model(g)
    srv = Server.for_model(m, slots=3, max_seq=192, pages=pages)
    reqs = []
    for i, (n, k) in enumerate([(40, 12), (70, 30), (9, 20), (100, 8), (33, 25)]):
        p = [int(t) for t in synth.prompt_ids(2048, n, seed=500 + i)]
        reqs.append((srv.submit(p, max_tokens=k), p, k))
    steps = 0
    while srv.busy() and steps < 400:
        srv.step()
        steps += 1
        if steps == 5:  # a late arrival while the first ones decode
            p = [int(t) for t in synth.prompt_ids(2048, 50, seed=599)]
            reqs.append((srv.submit(p, max_tokens=15), p, 15))
    assert not srv.busy()
    exact = total = 0
    for rid, p, k in reqs:
        got = [int(t) for t in srv.result(rid)]
        assert len(got) == k, rid
        exact += _check_greedy(o, p, got)
        total += k
    print(f"pages {pages}: {exact}/{total} tokens are the oracle's exact argmax; "
          f"{srv.steps} batched steps, {srv.preemptions} preemptions")
