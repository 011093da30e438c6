"""Dense matmul weights (GGUF F32, F16 and the reference's Q8_K) on the GPU
against the CPU oracle.

The reference dequantises every matmul weight to f32 (src/gguf/dequant.rs:
10-52, 201-232) and its own model fixtures are all-F32 GGUFs
(src/model/forward.rs:713). The first two tests rebuild those fixtures
(forward.rs:729-839: hidden 8, two 4-wide heads, ffn 16, vocab 100, ones or
zeros) and run what the reference's tests run (forward over one token,
generate 5 tokens after a 3-token prompt), held to the oracle. The others
load random-weight models of each dense type (head size 64) and compare the
prefill, decode steps, the non-causal forward and a batched decode step at
the logits bar |gpu - ref| <= 2e-2 + 1e-2 |ref|.
"""
import os

import numpy as np
import pytest

from gguf_builder import GgufBuilder, llama_meta
from inferox_b200 import Model, synth
from oracle import refcpu as R

pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-2, 1e-2
R.set_threads(os.cpu_count() or 8)


def _close(g, r):
    return np.all(np.abs(g - r) <= ATOL + RTOL * np.abs(r))


def _fixture(fill: float) -> bytes:
    """forward.rs:729-780 (fill 1.0) / :786-839 (fill 0.0): one layer of F32."""
    hs, inter, vocab = 8, 16, 100
    g = llama_meta(GgufBuilder(), vocab, hs, 1, 2, 2, inter, 128 if fill else 32)
    ones = np.ones(hs, np.float32)
    zv = np.zeros(vocab * hs, np.float32)
    sq = np.full(hs * hs, fill, np.float32)
    ih = np.full(inter * hs, fill, np.float32)
    g.tensor_f32("token_embd.weight", [100, hs], zv)
    g.tensor_f32("output_norm.weight", [hs], ones)
    g.tensor_f32("output.weight", [100, hs], zv)
    g.tensor_f32("blk.0.attn_norm.weight", [hs], ones)
    for n in ("attn_q", "attn_k", "attn_v", "attn_output"):
        g.tensor_f32(f"blk.0.{n}.weight", [hs, hs], sq)
    g.tensor_f32("blk.0.ffn_norm.weight", [hs], ones)
    g.tensor_f32("blk.0.ffn_gate.weight", [inter, hs], ih)
    g.tensor_f32("blk.0.ffn_up.weight", [inter, hs], ih)
    g.tensor_f32("blk.0.ffn_down.weight", [hs, inter], ih)
    return g.build()


def test_reference_fixture_forward():
    b = _fixture(1.0)
    m, o = Model.from_bytes(b), R.Model(b)
    got, ref = m.forward([0]), o.forward([0])
    assert got.shape == ref.shape and got.shape[-1] == 100  # forward.rs:779
    assert _close(got, ref), float(np.max(np.abs(got - ref)))


def test_reference_fixture_generate():
    b = _fixture(0.0)
    m, o = Model.from_bytes(b), R.Model(b)
    kv, okv = m.kv_cache(32), o.kv_cache(1, 32)
    got = m.generate([0, 1, 2], 5, kv)
    ref = o.generate([0, 1, 2], 5, okv)
    assert len(got) == 5 and all(int(t) < 100 for t in got)  # forward.rs:834-835
    assert len(kv) == 3 + 5  # forward.rs:836
    assert np.array_equal(np.asarray(got), np.asarray(ref))


V, D, L, H, G, F, CTX = 512, 256, 2, 4, 2, 512, 96


def _q8k_blocks(rng, n):
    """Random blocks of the reference's Q8_K (dequant.rs:210-232): d and dmin
    f16, 32 u8 scales (one per 8 values), 256 int8: y = d * sc * q - dmin."""
    out = bytearray()
    for _ in range(n // 256):
        out += np.float16(rng.uniform(1e-4, 3e-4)).tobytes()
        out += np.float16(rng.uniform(-2e-3, 2e-3)).tobytes()
        out += rng.integers(1, 9, 32, dtype=np.uint8).tobytes()
        out += rng.integers(-127, 128, 256, dtype=np.int64).astype(np.int8).tobytes()
    return bytes(out)


def _dense_model(ttype: int) -> bytes:
    rng = np.random.default_rng(40 + ttype)
    hd = D // H
    g = llama_meta(GgufBuilder(), V, D, L, H, G, F, CTX, rope_base=10000.0)

    def mat(name, rows, cols):
        if ttype == 15:
            g.tensor(name, [cols, rows], 15, _q8k_blocks(rng, rows * cols))
            return
        w = rng.normal(0.0, 0.02, rows * cols).astype(np.float32)
        if ttype == 1:
            g.tensor(name, [cols, rows], 1, w.astype(np.float16).tobytes())
        else:
            g.tensor_f32(name, [cols, rows], w)

    mat("token_embd.weight", V, D)
    g.tensor_f32("output_norm.weight", [D], rng.uniform(0.5, 1.5, D).astype(np.float32))
    mat("output.weight", V, D)
    for l in range(L):
        p = f"blk.{l}."
        g.tensor_f32(p + "attn_norm.weight", [D], rng.uniform(0.5, 1.5, D).astype(np.float32))
        mat(p + "attn_q.weight", D, D)
        mat(p + "attn_k.weight", G * hd, D)
        mat(p + "attn_v.weight", G * hd, D)
        mat(p + "attn_output.weight", D, D)
        g.tensor_f32(p + "ffn_norm.weight", [D], rng.uniform(0.5, 1.5, D).astype(np.float32))
        mat(p + "ffn_gate.weight", F, D)
        mat(p + "ffn_up.weight", F, D)
        mat(p + "ffn_down.weight", D, F)
    return g.build()


@pytest.mark.parametrize("ttype", [0, 1, 15])  # F32, F16, Q8_K
def test_dense_weights_match_oracle(ttype):
    b = _dense_model(ttype)
    m, o = Model.from_bytes(b), R.Model(b)
    prompt = synth.prompt_ids(V, 24, seed=ttype)
    kv, okv = m.kv_cache(64), o.kv_cache(L, 64)
    gl, rl = m.prefill(prompt, kv), o.prefill(prompt, okv)
    assert _close(gl, rl), float(np.max(np.abs(gl - rl)))
    tok = R.argmax(rl[-1])
    for i in range(6):
        gl, rl = m.decode_step(tok, kv), o.decode_step(tok, okv)
        assert _close(gl, rl), (i, float(np.max(np.abs(gl - rl))))
        tok = R.argmax(rl)
    assert kv.decode_kernels() > 1  # the per-op dense kernels, not the persistent one
    fg, fr = m.forward(prompt[:10]), o.forward(prompt[:10])
    assert _close(fg, fr), float(np.max(np.abs(fg - fr)))
    # two sequences decoded together (the batched step's small GEMM path)
    kb = m.kv_batch(2, 64)
    toks = []
    for s in range(2):
        p = synth.prompt_ids(V, 12, seed=100 + s)
        okv = o.kv_cache(L, 64)
        r = o.prefill(p, okv, True)[0]
        assert _close(kb.prefill(s, p, True)[0], r)
        t = R.argmax(r)
        toks.append((t, okv))
    got, _ = kb.decode_step([t for t, _ in toks])
    for s, (t, okv) in enumerate(toks):
        r = o.decode_step(t, okv)
        assert _close(got[s], r), (s, float(np.max(np.abs(got[s] - r))))
