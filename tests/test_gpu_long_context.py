"""Parity at the benchmarked context lengths.

The benchmark prefills 1024 (8B) or 2048 (70B) prompt tokens and then
decodes at contexts above a thousand positions. These tests hold exactly
those code paths to the CPU oracle on narrow two-layer models whose head
geometry matches the benchmark shapes, so the oracle still finishes in
seconds:

* 8B geometry: head_dim 128, 4 query heads per kv head, 8 kv heads. With a
  cache of ~1100 rows the persistent kernel cuts each kv head's rows into
  18 splits, as in the 8B benchmark, so the one-round-trip split combine
  and the tensor-core attention items run at the benchmark's split sizes.
* 70B geometry: head_dim 128, 8 query heads per kv head (the FMA attention
  loops and the general split combine), a 2048-token prompt.
* 1B geometry: head_dim 64, tied Q6_K embedding / output, 2048 tokens.

The prompt goes through the prefill path (tcgen05 GEMM over 1024-2048
token rows, tensor-core causal attention over 16-32 query tiles); the K/V
cache it leaves is compared with the oracle's; then 40 teacher-forced
decode steps run on the persistent kernel at contexts above 1024.

Bar (the north star's): logits within |gpu - ref| <= 2e-2 + 1e-2 |ref|,
teacher-forced top-1 agreement on at least 99% of the steps. The cache is
held to the oracle's f32 values: layer 0 within the f16 rounding of the
device cache plus the matmul difference (2e-3 absolute + 2e-3 relative, as
in the short tests); the last layer within 8e-3 absolute + 4e-3 relative,
because its K and V also carry the difference of the prefill attention
below it, which multiplies f16 Q, K, V and probabilities where the
reference uses f32 (about 1e-3 relative of the attention output at these
contexts; measured 5e-3 absolute on the 8B geometry's second layer). The
worst cache and logit differences are printed.
Reference: src/model/forward.rs:215-337 (prefill, chunk attention),
:344-440 (decode attention over the cache), :543-586 (decode step).
"""
import os

import numpy as np
import pytest

from inferox_b200 import Model, synth
from oracle import refcpu as R

pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-2, 1e-2
R.set_threads(os.cpu_count() or 8)

CASES = {
    "8b_geometry": (dict(vocab=4096, dim=4096, n_layers=2, n_heads=32, n_kv_heads=8, ffn=4096,
                         context=4096, rope_base=500000.0, mix=1, seed=11), 1024),
    "70b_geometry": (dict(vocab=4096, dim=2048, n_layers=2, n_heads=16, n_kv_heads=2, ffn=2048,
                          context=4096, rope_base=10000.0, mix=1, seed=12), 2048),
    "1b_geometry": (dict(vocab=8192, dim=1024, n_layers=2, n_heads=16, n_kv_heads=4, ffn=2048,
                         context=4096, rope_base=500000.0, mix=1, tied=1, seed=13), 2048),
}
STEPS = 40


def _close(g, r):
    return np.all(np.abs(g - r) <= ATOL + RTOL * np.abs(r))


@pytest.mark.parametrize("case", sorted(CASES))
def test_long_prompt_then_decode(case):
    kw, n_prompt = CASES[case]
    g = synth.build(None, **kw)
    m, o = Model.from_bytes(g), R.Model(g)
    L, V = int(m.config.n_layers), int(m.config.vocab_size)
    max_seq = n_prompt + STEPS + 40
    prompt = synth.prompt_ids(V, n_prompt, seq_index=7)
    kv, okv = m.kv_cache(max_seq), o.kv_cache(L, max_seq)
    gl = m.prefill(prompt, kv, True)[0]
    rl = o.prefill(prompt, okv, True)[0]
    assert _close(gl, rl), float(np.max(np.abs(gl - rl)))
    # the cache the long prefill wrote (every position, both ends of the stack)
    assert len(kv) == len(okv) == n_prompt
    for layer in (0, L - 1):
        atol, rtol = (2e-3, 2e-3) if layer == 0 else (8e-3, 4e-3)
        for which_v in (False, True):
            a, b = kv.read(layer, which_v), okv.read(layer, which_v)
            assert a.shape == b.shape == (n_prompt, okv.kv_dim)
            print(f"{case} layer {layer} {'V' if which_v else 'K'}: max |d| {np.max(np.abs(a - b)):.2e}")
            assert np.allclose(a, b, atol=atol, rtol=rtol), (layer, which_v, float(np.max(np.abs(a - b))))
    agree = int(R.argmax(gl) == R.argmax(rl))
    tok = R.argmax(rl)
    worst = 0.0
    for i in range(STEPS):
        gl, rl = m.decode_step(tok, kv), o.decode_step(tok, okv)
        worst = max(worst, float(np.max(np.abs(gl - rl))))
        assert _close(gl, rl), (i, worst)
        agree += int(R.argmax(gl) == R.argmax(rl))
        tok = R.argmax(rl)
    print(f"{case}: worst decode logit |d| {worst:.2e}, top-1 agreement {agree}/{STEPS + 1}")
    assert agree >= 0.99 * (STEPS + 1), (agree, STEPS + 1)
    assert kv.decode_kernels() == 1  # the persistent decode kernel ran these steps
    # decode appended rows n_prompt .. n_prompt + STEPS - 1 of the cache
    a, b = kv.read(L - 1, True), okv.read(L - 1, True)
    assert np.allclose(a, b, atol=8e-3, rtol=4e-3), float(np.max(np.abs(a - b)))


def test_long_greedy_matches_stepping():
    """The device-fed greedy loop (one persistent launch per token, the argmax
    fed back on the device, as the benchmark times it) produces the tokens
    that stepping with the host reading each argmax produces, at contexts
    above 1024 on the 8B geometry."""
    kw, n_prompt = CASES["8b_geometry"]
    g = synth.build(None, **kw)
    m = Model.from_bytes(g)
    V = int(m.config.vocab_size)
    prompt = synth.prompt_ids(V, n_prompt, seq_index=8)
    ka, kb = m.kv_cache(n_prompt + 64), m.kv_cache(n_prompt + 64)
    first = int(np.argmax(m.prefill(prompt, ka, True)[0]))
    assert first == int(np.argmax(m.prefill(prompt, kb, True)[0]))
    toks, _ = m.decode_greedy(first, 24, ka)
    tok = first
    for i in range(24):
        lg = m.decode_step(tok, kb)
        tok = R.argmax(lg)
        if int(toks[i]) != tok:
            # rows split across CTAs are summed with float atomics, so two runs
            # of one step agree to a few ulps: a divergence must be a near tie
            gap = abs(float(lg[tok]) - float(lg[int(toks[i])]))
            assert gap <= 1e-3, (i, gap)
            break


def test_short_context_in_large_cache():
    """A 512-token context in a 4096-position cache: the persistent kernel
    splits each kv head's attention by the context's length (18 splits of
    ~29 rows) rather than by the cache's (52), so the combine and the item
    count follow the context; logits held to the oracle as above."""
    kw, _ = CASES["70b_geometry"]
    g = synth.build(None, **kw)
    m, o = Model.from_bytes(g), R.Model(g)
    L, V = int(m.config.n_layers), int(m.config.vocab_size)
    n_prompt, steps = 512, 24
    prompt = synth.prompt_ids(V, n_prompt, seq_index=9)
    kv, okv = m.kv_cache(4096), o.kv_cache(L, 4096)
    gl = m.prefill(prompt, kv, True)[0]
    rl = o.prefill(prompt, okv, True)[0]
    assert _close(gl, rl), float(np.max(np.abs(gl - rl)))
    agree = int(R.argmax(gl) == R.argmax(rl))
    tok = R.argmax(rl)
    worst = 0.0
    for i in range(steps):
        gl, rl = m.decode_step(tok, kv), o.decode_step(tok, okv)
        worst = max(worst, float(np.max(np.abs(gl - rl))))
        assert _close(gl, rl), (i, worst)
        agree += int(R.argmax(gl) == R.argmax(rl))
        tok = R.argmax(rl)
    print(f"short context in a large cache: worst decode logit |d| {worst:.2e}, top-1 {agree}/{steps + 1}")
    assert agree >= 0.99 * (steps + 1), (agree, steps + 1)
    assert kv.decode_kernels() == 1
