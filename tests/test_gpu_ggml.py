"""A llama.cpp-written GGUF (ggml type ids and block orders, int8 Q6_K scales
of both signs) loaded with kquant_layout="ggml", against the CPU oracle.

The file is written by llama.cpp's own writer (gguf-py's GGUFWriter): Q8_0
blocks from gguf-py's quantiser under ggml's id 8 for ffn_up beside a Q4_K
ffn_gate (a unit width of 128 beside 256, so the fused gate/up GEMV runs as
two plans); Q4_K weights quantised by the library and rewritten in ggml's
nibble order, Q6_K weights from a quantiser that gives each 16-element
group a scale of random sign (as llama.cpp's own quantiser does) — gguf-py
has no K-quant quantiser, so these blocks are checked by decoding them with
gguf-py. The oracle runs the same weights decoded by gguf-py's dequantiser
(llama.cpp's formulas) and stored as F32 tensors, so the
comparison covers the load-time permutation, the int8 scale reading in the
GEMV (persistent decode kernel), the tcgen05 prefill GEMM, the small-batch
GEMM and the embedding gather, at the logits bar |gpu - ref| <= 2e-2 +
1e-2 |ref|. A tied variant takes token_embd from Q6_K (the embedding
gather and the output projection both read int8 scales).
"""
import os
import tempfile

import numpy as np
import pytest

from gguf_builder import GgufBuilder, llama_meta
from inferox_b200 import IfxError, Model, synth

gguf = pytest.importorskip("gguf")
from gguf import quants as ggq  # noqa: E402
from oracle import ggml_ref as G
from oracle import refcpu as R

pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-2, 1e-2
R.set_threads(os.cpu_count() or 8)
V, D, L, H, KVH, F, CTX = 1024, 512, 2, 8, 2, 1024, 96


def _close(g, r):
    return np.all(np.abs(g - r) <= ATOL + RTOL * np.abs(r))


def _models(tied: bool):
    rng = np.random.default_rng(17 + tied)
    hd = D // H
    mats = []  # (name, rows, cols, ggml type)
    emb_type = 14 if tied else 12
    mats.append(("token_embd.weight", V, D, emb_type))
    if not tied:
        mats.append(("output.weight", V, D, 14))
    for l in range(L):
        p = f"blk.{l}."
        mats += [(p + "attn_q.weight", D, D, 12), (p + "attn_k.weight", KVH * hd, D, 12),
                 (p + "attn_v.weight", KVH * hd, D, 14), (p + "attn_output.weight", D, D, 12),
                 (p + "ffn_gate.weight", F, D, 12), (p + "ffn_up.weight", F, D, 8),
                 (p + "ffn_down.weight", D, F, 14 if l % 2 == 0 else 12)]
    g_f32 = llama_meta(GgufBuilder(), V, D, L, H, KVH, F, CTX, rope_base=500000.0)
    w = gguf.GGUFWriter(path=None, arch="llama")
    w.add_uint32("llama.vocab_size", V)
    w.add_uint32("llama.embedding_length", D)
    w.add_uint32("llama.block_count", L)
    w.add_uint32("llama.attention.head_count", H)
    w.add_uint32("llama.attention.head_count_kv", KVH)
    w.add_uint32("llama.feed_forward_length", F)
    w.add_float32("llama.attention.layer_norm_rms_epsilon", 1e-5)
    w.add_uint32("llama.context_length", CTX)
    w.add_float32("llama.rope.freq_base", 500000.0)
    norms = {"output_norm.weight": D}
    for l in range(L):
        norms[f"blk.{l}.attn_norm.weight"] = D
        norms[f"blk.{l}.ffn_norm.weight"] = D
    for name, n in norms.items():
        v = (1.0 + rng.normal(0, 0.05, n)).astype(np.float32)
        w.add_tensor(name, v)
        g_f32.tensor_f32(name, [n], v)
    for name, rows, cols, t in mats:
        x = rng.normal(0, 0.02, rows * cols).astype(np.float32)
        if t == 12:
            raw = np.frombuffer(G.q4k_reference_to_ggml(synth.quantize(12, x)), np.uint8)
        elif t == 14:
            raw = np.frombuffer(G.quantize_q6k_ggml(x, rng), np.uint8)
        else:
            raw = ggq.quantize(x.reshape(rows, cols), gguf.GGMLQuantizationType.Q8_0).reshape(-1)
        qt = gguf.GGMLQuantizationType(t)
        w.add_tensor(name, raw.reshape(rows, -1), raw_dtype=qt)
        vals = ggq.dequantize(raw.reshape(rows, -1), qt).reshape(-1).astype(np.float32)
        assert np.array_equal(vals, G.dequant(t, raw))  # the restatement agrees
        g_f32.tensor_f32(name, [cols, rows], vals)
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "llama.gguf")
        w.path = path
        w.write_header_to_file(path=path)
        w.write_kv_data_to_file()
        w.write_tensors_to_file()
        w.close()
        data = open(path, "rb").read()
    return np.frombuffer(data, np.uint8), g_f32.build()


@pytest.mark.parametrize("tied", [False, True])
def test_ggml_file_matches_oracle(tied):
    raw, f32 = _models(tied)
    m = Model.from_bytes(raw, kquant_layout="ggml")
    o = R.Model(f32)
    prompt = synth.prompt_ids(V, 37, seed=3)
    kv, okv = m.kv_cache(CTX), o.kv_cache(L, CTX)
    gl = m.prefill(prompt, kv, True)[0]
    rl = o.prefill(prompt, okv, True)[0]
    assert _close(gl, rl), float(np.max(np.abs(gl - rl)))
    tok = R.argmax(rl)
    for _ in range(4):
        gl = m.decode_step(tok, kv)
        rl = o.decode_step(tok, okv)
        assert _close(gl, rl), float(np.max(np.abs(gl - rl)))
        tok = R.argmax(rl)
    assert kv.decode_kernels() == 1  # the persistent decode kernel ran
    # batched decode: the small-batch GEMM reads the same weights
    kb = m.kv_batch(2, 64)
    okv2 = [o.kv_cache(L, 64) for _ in range(2)]
    toks = []
    for b in range(2):
        p = prompt[: 9 + 4 * b]
        gl = kb.prefill(b, p, True)[0]
        rl = o.prefill(p, okv2[b], True)[0]
        assert _close(gl, rl)
        toks.append(R.argmax(rl))
    logits, _ = kb.decode_step(toks)
    for b in range(2):
        assert _close(logits[b], o.decode_step(toks[b], okv2[b]))


def test_ggml_file_needs_the_option():
    raw, _ = _models(False)
    with pytest.raises(IfxError):  # id 8 is Q8_1 to the reference: not a kernel type
        Model.from_bytes(raw)
    with pytest.raises(ValueError):
        Model.from_bytes(raw, kquant_layout="gguf")
