"""Prefill in chunks onto a non-empty cache, contiguous and paged, against
the CPU oracle.

The reference prefills a chunk with attention inside the chunk only and
RoPE positions 0..n regardless of the cache start (src/model/forward.rs:
243-244, 246-253, 266-274); the K/V rows land at cache_start + t. Here two
chunks (100 then 77 tokens: the second starts inside a 64-position page
and a 64-key tile) go into one cache, for every query-heads-per-kv-head
ratio the streamed prefill attention kernel takes (1, 2, 4, 8 heads per
kv head; head sizes 64 and 128), then decode steps read the whole cache.
Logits are held to the oracle at |gpu - ref| <= 2e-2 + 1e-2 |ref| and the
cached K/V rows to the oracle's cache.
"""
import os

import numpy as np
import pytest

from inferox_b200 import Model, synth
from oracle import refcpu as R

pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-2, 1e-2
R.set_threads(os.cpu_count() or 8)


def _close(g, r):
    return np.all(np.abs(g - r) <= ATOL + RTOL * np.abs(r))


CASES = {  # name: (heads, kv_heads, head size)
    "grp1_hd128": (4, 4, 128),
    "grp2_hd128": (8, 4, 128),
    "grp4_hd64": (8, 2, 64),
    "grp8_hd64": (16, 2, 64),
}


def _model(name):
    h, kvh, hd = CASES[name]
    return synth.build(None, vocab=1024, dim=h * hd, n_layers=2, n_heads=h, n_kv_heads=kvh,
                       ffn=512, context=256, rope_base=10000.0, mix=1,
                       seed=7 + sorted(CASES).index(name))


@pytest.mark.parametrize("name", sorted(CASES))
def test_two_chunks_then_decode(name):
    g = _model(name)
    m, o = Model.from_bytes(g), R.Model(g)
    L = int(m.config.n_layers)
    a = synth.prompt_ids(1024, 100, seed=1)
    b = synth.prompt_ids(1024, 77, seed=2)
    kv, okv = m.kv_cache(256), o.kv_cache(L, 256)
    assert _close(m.prefill(a, kv), o.prefill(a, okv))
    gl, rl = m.prefill(b, kv), o.prefill(b, okv)
    assert _close(gl, rl), float(np.max(np.abs(gl - rl)))
    assert len(kv) == 177
    tok = R.argmax(rl[-1])
    for i in range(3):
        gl, rl = m.decode_step(tok, kv), o.decode_step(tok, okv)
        assert _close(gl, rl), (i, float(np.max(np.abs(gl - rl))))
        tok = R.argmax(rl)
    for layer in range(L):  # the f16 cache against the oracle's f32 one
        atol, rtol = (2e-3, 2e-3) if layer == 0 else (8e-3, 4e-3)
        for v in (False, True):
            gc, rc = kv.read(layer, v), okv.read(layer, v)
            assert np.allclose(gc, rc, atol=atol, rtol=rtol), (layer, v, float(np.max(np.abs(gc - rc))))


@pytest.mark.parametrize("name", ["grp4_hd64", "grp1_hd128"])
def test_two_chunks_paged(name):
    g = _model(name)
    m, o = Model.from_bytes(g), R.Model(g)
    L = int(m.config.n_layers)
    kb = m.kv_batch(2, 256, pages=12)
    a = synth.prompt_ids(1024, 100, seed=3)
    b = synth.prompt_ids(1024, 77, seed=4)
    okv = o.kv_cache(L, 256)
    o.prefill(a, okv)
    kb.prefill(1, a)
    gl, rl = kb.prefill(1, b), o.prefill(b, okv)
    assert _close(gl, rl), float(np.max(np.abs(gl - rl)))
