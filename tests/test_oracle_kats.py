"""Pins the CPU oracle (oracle/refcpu.c) against every known-answer test the
reference's own sources hold. Each test names the reference test it ports.

The reference is Rust and cannot be built here, so these KATs are what pins
the oracle; the GPU parity tests then compare the CUDA path to this oracle.
"""
import struct

import numpy as np
import pytest

from gguf_builder import GgufBuilder, llama_meta
from oracle import refcpu as R


def f16b(v: float) -> bytes:
    return np.float16(v).tobytes()


# ---------------- dequant.rs tests (dequant.rs:247-392) -------------------

def test_dequantize_q4_0_single_block():  # dequant.rs:247-267
    block = f16b(0.5) + bytes(((j << 4) | j) for j in range(16))
    out = R.dequantize(R.Q4_0, block, 32)
    for j, v in enumerate(out):
        assert abs(v - ((j % 16) - 8) * 0.5) < 1e-6


def test_dequantize_q8_0_single_block():  # dequant.rs:269-287
    block = f16b(0.25) + bytes(range(32))
    out = R.dequantize(R.Q8_0, block, 32)
    for j, v in enumerate(out):
        assert abs(v - j * 0.25) < 1e-6


def test_dequantize_f16_to_f32():  # dequant.rs:289-298
    data = b"".join(f16b(v) for v in (1.0, 2.0, -3.0))
    assert list(R.dequantize(R.F16, data, 3)) == [1.0, 2.0, -3.0]


def test_dequantize_f32_identity():  # dequant.rs:300-309
    data = np.array([1.0, 2.0, -3.0], np.float32).tobytes()
    assert list(R.dequantize(R.F32, data, 3)) == [1.0, 2.0, -3.0]


def test_dequantize_q4_k_single_block():  # dequant.rs:311-337
    block = bytearray(f16b(1.0) + f16b(0.0))
    block += bytes([1, 1, 1, 1, 0, 0, 0, 0, 1, 1, 1, 1])
    for _ in range(8):
        for pair in range(16):
            low = 2 * pair
            high = (2 * pair + 1) % 32
            block.append(((high << 4) & 0xFF) | low)  # u8 shift wraps in Rust
    out = R.dequantize(R.Q4_K, bytes(block), 256)
    for j, v in enumerate(out):
        assert abs(v - float((j % 32) % 16)) < 1e-6, j


def test_dequantize_q6_k_single_block():  # dequant.rs:339-359
    block = f16b(1.0) + bytes([1] * 16) + bytes(128) + bytes([0b10101010] * 64)
    out = R.dequantize(R.Q6_K, block, 256)
    assert np.all(np.abs(out) < 1e-6)


def test_dequantize_q8_k_single_block():  # dequant.rs:361-382
    block = f16b(1.0) + f16b(0.0) + bytes([1] * 32) + bytes((j & 0xFF) for j in range(256))
    out = R.dequantize(R.Q8_K, block, 256)
    for j, v in enumerate(out):
        assert abs(v - float(np.int8(np.uint8(j)))) < 1e-6


def test_unsupported_type_fails():  # dequant.rs:384-392
    with pytest.raises(R.OracleError) as e:
        R.dequantize(R.Q5_0, bytes(22), 32)
    assert e.value.name == "UnknownTensorType"


def test_dequantize_wrong_size_is_eof():  # dequantize_f32 size check, dequant.rs:14-16
    with pytest.raises(R.OracleError) as e:
        R.dequantize(R.Q8_0, bytes(33), 32)
    assert e.value.name == "UnexpectedEof"


# Our own Q6_K KATs: the element order and the u8 reading of the scale byte
# (dequant.rs:189-196) are not pinned by the reference's tests.
def test_q6_k_element_order_and_u8_scale():
    d = 0.5
    scales = bytes([(3 * g + 1) & 0xFF for g in range(15)] + [0xFF])  # last byte 255, not -1
    rng = np.random.default_rng(7)
    q = rng.integers(0, 64, 256)
    ql = bytearray(128)
    qh = bytearray(64)
    for j in range(256):
        nib = q[j] & 15
        ql[j // 2] |= nib if j % 2 == 0 else nib << 4
        qh[j // 4] |= ((q[j] >> 4) & 3) << (2 * (j % 4))
    block = f16b(d) + scales + bytes(ql) + bytes(qh)
    out = R.dequantize(R.Q6_K, block, 256)
    for j in range(256):
        exp = np.float32(np.float32(d) * np.float32(scales[j // 16])) * np.float32(q[j] - 32)
        assert out[j] == exp, j


def test_q4_k_scale_min_unpack_high_groups():
    # groups 4..7 take 4 low bits from scales[g+4] and 2 high bits from
    # scales[g-4] (sc) / scales[g] (mn): dequant.rs:146-147.
    sc = [5, 17, 33, 63, 44, 60, 1, 38]
    mn = [2, 63, 7, 19, 50, 3, 61, 16]
    s = bytearray(12)
    for g in range(4):
        s[g] = sc[g] | ((sc[g + 4] >> 4) << 6)
        s[g + 4] = mn[g] | ((mn[g + 4] >> 4) << 6)
        s[g + 8] = (sc[g + 4] & 15) | ((mn[g + 4] & 15) << 4)
    qs = bytes([0x21] * 128)  # even l -> 1, odd l -> 2
    block = f16b(0.25) + f16b(0.125) + bytes(s) + qs
    out = R.dequantize(R.Q4_K, block, 256)
    for g in range(8):
        dall = np.float32(0.25) * np.float32(sc[g])
        dm = np.float32(0.125) * np.float32(mn[g])
        for l in range(32):
            qv = 1 if l % 2 == 0 else 2
            assert out[g * 32 + l] == np.float32(dall * np.float32(qv)) - dm


def test_f16_subnormal_and_specials():
    assert R.f16_to_f32(0x0001) == 2.0 ** -24
    assert R.f16_to_f32(0x3C00) == 1.0
    assert R.f16_to_f32(0xC000) == -2.0
    assert R.f16_to_f32(0x7C00) == float("inf")
    assert np.isnan(R.f16_to_f32(0x7E00))
    for h in range(0, 65536, 97):
        exp = np.frombuffer(struct.pack("<H", h), np.float16)[0].astype(np.float32)
        got = np.float32(R.f16_to_f32(h))
        assert (np.isnan(exp) and np.isnan(got)) or exp == got
    # NaN: payload kept, quiet bit set (half 2.x f16_to_f32)
    b = np.array([R.f16_to_f32(0x7C01)], np.float32).view(np.uint32)[0]
    assert b == (0x7FC00000 | (1 << 13))
    b = np.array([R.f16_to_f32(0xFE00)], np.float32).view(np.uint32)[0]
    assert b == (0x80000000 | 0x7FC00000 | (0x200 << 13))


# ---------------- ops.rs tests (ops.rs:293-416) ----------------------------

def test_matmul_2x3x4():  # ops.rs:293-314
    a = [1, 2, 3, 4, 5, 6]
    b = [1, 0, 1, 0, 0, 1, 0, 1, 1, 1, 0, 0]
    c = R.matmul(a, b, 2, 4, 3)
    assert list(c[:4]) == [4, 5, 1, 2]
    assert list(c[4:]) == [10, 11, 4, 5]


def test_matmul_t_matches_transpose():  # ops.rs:316-327
    assert list(R.matmul_t([1, 2, 3, 4], [0, 1, 2, 3], 2, 2, 2)) == [2, 8, 4, 18]


def test_matmul_with_non_multiple_of_eight():  # ops.rs:329-337
    assert list(R.matmul([1, 2, 3], [1, 0, 2, 1, 0, 2], 1, 2, 3)) == [5, 8]


def test_matmul_t_with_non_multiple_of_eight():  # ops.rs:339-346
    assert list(R.matmul_t([1, 2, 3], [1, 0, 2, 2, 1, 0], 1, 2, 3)) == [7, 4]


def test_rms_norm_unit_scale():  # ops.rs:348-357
    x = R.rms_norm([1, 2, 3, 4], [1] * 4, 1e-5)
    ms = np.float32(7.5)
    scale = np.float32(1.0) / np.sqrt(ms + np.float32(1e-5), dtype=np.float32)
    assert list(x) == [np.float32(v) * scale for v in (1, 2, 3, 4)]


def test_rms_norm_with_weight():  # ops.rs:359-369
    w = [0.5, 1.0, 1.5, 2.0]
    x = R.rms_norm([2, 2, 2, 2], w, 1e-5)
    assert np.all(np.abs(x - np.array(w, np.float32)) < 1e-5)


def _sigmoid(v):
    v = np.float32(min(max(v, -80.0), 80.0))
    return np.float32(1.0) / (np.float32(1.0) + np.exp(-v, dtype=np.float32))


def test_silu_values():  # ops.rs:371-380
    x = R.silu([0.0, 1.0, -1.0, 2.0])
    assert abs(x[0]) < 1e-6
    assert abs(x[1] - 1.0 * _sigmoid(1.0)) < 1e-6
    assert abs(x[2] + _sigmoid(-1.0)) < 1e-6
    assert abs(x[3] - 2.0 * _sigmoid(2.0)) < 1e-6


def test_swiglu_elementwise():  # ops.rs:382-394
    g, u = [0.0, 1.0, -1.0], [2.0, 3.0, 4.0]
    o = R.swiglu(g, u)
    for i in range(3):
        assert abs(o[i] - g[i] * _sigmoid(g[i]) * u[i]) < 1e-6


def test_add_in_place_works():  # ops.rs:396-401
    assert list(R.add_in_place([1, 2, 3], [0.5, 1.0, 1.5])) == [1.5, 3.0, 4.5]


def test_softmax_rows_sums_to_one():  # ops.rs:403-416
    x = R.softmax_rows([1, 2, 3, 0, 0, 0], 2, 3)
    assert abs(x[:3].sum() - 1) < 1e-5 and abs(x[3:].sum() - 1) < 1e-5
    assert x[2] > x[1] > x[0]


def test_embedding_lookup_oob_is_error():  # ops.rs:252-255 (panic -> error code)
    with pytest.raises(R.OracleError):
        R.embedding_lookup(np.zeros(8), [2], 4)


def test_avx2_intrinsics_match_scalar_lane_emulation():
    rng = np.random.default_rng(3)
    for k in (1, 7, 8, 9, 31, 64, 300):
        a = rng.standard_normal(3 * k).astype(np.float32)
        b = rng.standard_normal(5 * k).astype(np.float32)
        assert np.array_equal(R.matmul_t(a, b, 3, 5, k), R.matmul_t(a, b, 3, 5, k, emul=True))


def test_rope_position_zero_is_identity():  # ops.rs:270-286 at seq_len=1
    x = np.random.default_rng(0).standard_normal(2 * 8).astype(np.float32)
    assert np.array_equal(R.rope(x, 1, 2, 8, 8, 10000.0), x)


def test_argmax_last_index_on_ties():  # forward.rs:615-622 (Iterator::max_by)
    assert R.argmax([1.0, 3.0, 3.0, 2.0]) == 2
    assert R.argmax([0.0] * 5) == 4


# ---------------- sampler.rs tests (sampler.rs:88-123) ---------------------

def test_greedy_picks_highest():  # sampler.rs:88-94
    assert R.sample([1.0, 3.0, 2.0], 0.0, 0, 1.0, 0.5) == 1


def test_temperature_non_greedy_samples_from_distribution():  # sampler.rs:96-108
    for u in np.linspace(0, 0.999, 17):
        assert R.sample([0.0, 1.0, 0.0], 1.0, 0, 1.0, float(u)) < 3


def test_top_k_truncates():  # sampler.rs:110-123
    for u in np.linspace(0, 0.999, 17):
        assert R.sample([10.0, 1.0, 1.0, 1.0], 1.0, 2, 1.0, float(u)) <= 1


def test_weighted_index_partition_point():
    # probabilities after softmax of [0, ln3] at T=1 are [0.25, 0.75]:
    # u < 0.25 picks 0, above picks 1.
    lg = [0.0, float(np.log(3.0))]
    assert R.sample(lg, 1.0, 0, 1.0, 0.1) == 0
    assert R.sample(lg, 1.0, 0, 1.0, 0.3) == 1


def test_top_p_cutoff():
    # sorted probs ~[0.64, 0.24, 0.09, 0.03]; top_p 0.8 keeps 2 tokens.
    lg = [3.0, 2.0, 1.0, -0.1]
    for u in np.linspace(0, 0.999, 23):
        assert R.sample(lg, 1.0, 0, 0.8, float(u)) in (0, 1)


# ---------------- GGUF / weights tests ------------------------------------

def test_opens_and_reads_tensor_bytes():  # weights.rs:150-169
    g = GgufBuilder()
    g.tensor_f32("token_embeddings", [2], [1.5, 2.5])
    f = R.GgufFile(g.build())
    assert f.n_tensors() == 1
    assert list(np.frombuffer(f.tensor("token_embeddings"), np.float32)) == [1.5, 2.5]


def test_tensor_not_found_returns_error():  # weights.rs:171-183
    g = GgufFile_simple()
    with pytest.raises(R.OracleError) as e:
        g.tensor("missing")
    assert e.value.name == "TensorNotFound"


def GgufFile_simple():
    g = GgufBuilder()
    g.tensor_f32("token_embeddings", [2], [1.5, 2.5])
    return R.GgufFile(g.build())


def test_gguf_header_errors():  # file.rs:71-91, tensor.rs:52-54
    with pytest.raises(R.OracleError) as e:
        R.GgufFile(b"GGUX" + bytes(20))
    assert e.value.name == "InvalidMagic"
    with pytest.raises(R.OracleError) as e:
        R.GgufFile(b"GGUF" + struct.pack("<IQQ", 4, 0, 0))
    assert e.value.name == "UnsupportedVersion"
    g = GgufBuilder()
    g.tensor("t", [1, 1, 1, 1, 1], 0, bytes(4))
    with pytest.raises(R.OracleError) as e:
        R.GgufFile(g.build())
    assert e.value.name == "InvalidShape"
    g = GgufBuilder()
    g.raw_kv("k", 13, b"")
    with pytest.raises(R.OracleError) as e:
        R.GgufFile(g.build())
    assert e.value.name == "UnknownValueType"
    g = GgufBuilder()
    g.tensor("t", [4], 4, bytes(4))  # type id 4 does not exist
    with pytest.raises(R.OracleError) as e:
        R.GgufFile(g.build())
    assert e.value.name == "UnknownTensorType"
    with pytest.raises(R.OracleError) as e:
        R.GgufFile(b"GGUF" + struct.pack("<I", 3))
    assert e.value.name == "Io"


def test_truncated_tensor_data_is_eof():  # weights.rs:107-110
    g = GgufBuilder()
    g.tensor_f32("t", [4], [1, 2, 3, 4])
    data = g.build()[:-4]
    with pytest.raises(R.OracleError) as e:
        R.GgufFile(data).tensor("t")
    assert e.value.name == "UnexpectedEof"


def _test_llama_gguf() -> bytes:  # model/mod.rs:136-195
    g = GgufBuilder()
    llama_meta(g, 100, 64, 2, 4, 2, 128, 512)
    names = ["token_embd.weight", "output_norm.weight", "output.weight"]
    for i in range(2):
        names += [f"blk.{i}.{s}.weight" for s in (
            "attn_norm", "attn_q", "attn_k", "attn_v", "attn_output",
            "ffn_norm", "ffn_gate", "ffn_up", "ffn_down")]
    g.pad_between = False
    for n in names:
        g.tensors.append((n, [1, 1], 0, b""))
    raw = bytearray(g.build())
    raw += bytes(len(names) * 4 * 4)
    return bytes(raw)


def test_config_parsed_from_metadata():  # model/mod.rs:197-218
    m = R.Model(_test_llama_gguf())
    c = m.config
    assert c.architecture == b"llama"
    assert (c.vocab_size, c.hidden_size, c.n_layers, c.n_heads, c.n_kv_heads) == (100, 64, 2, 4, 2)
    assert c.head_dim == 16 and c.intermediate_size == 128 and c.context_length == 512
    assert abs(c.norm_eps - 1e-5) < 1e-10


def test_model_wires_layers_and_embeddings():  # model/mod.rs:220-238
    m = R.Model(_test_llama_gguf())
    assert m.has_output()
    assert m.config.n_layers == 2


def test_unsupported_architecture():  # config.rs:40-42
    g = GgufBuilder()
    g.string("general.architecture", "gpt2")
    with pytest.raises(R.OracleError) as e:
        R.Model(g.build())
    assert e.value.name == "UnsupportedArchitecture"


# ---------------- forward.rs tests (forward.rs:729-839) --------------------

def _tiny_f32_model(fill_qkvo: float, fill_ffn: float, ctx: int) -> bytes:
    hs, inter = 8, 16
    g = GgufBuilder()
    llama_meta(g, 100, hs, 1, 2, 2, inter, ctx)
    g.tensor_f32("token_embd.weight", [100, hs], np.zeros(100 * hs))
    g.tensor_f32("output_norm.weight", [hs], np.ones(hs))
    g.tensor_f32("output.weight", [100, hs], np.zeros(100 * hs))
    g.tensor_f32("blk.0.attn_norm.weight", [hs], np.ones(hs))
    for s in ("attn_q", "attn_k", "attn_v", "attn_output"):
        g.tensor_f32(f"blk.0.{s}.weight", [hs, hs], np.full(hs * hs, fill_qkvo))
    g.tensor_f32("blk.0.ffn_norm.weight", [hs], np.ones(hs))
    g.tensor_f32("blk.0.ffn_gate.weight", [inter, hs], np.full(inter * hs, fill_ffn))
    g.tensor_f32("blk.0.ffn_up.weight", [inter, hs], np.full(inter * hs, fill_ffn))
    g.tensor_f32("blk.0.ffn_down.weight", [hs, inter], np.full(inter * hs, fill_ffn))
    return g.build()


def test_layer_forward_runs_without_panic():  # forward.rs:729-784
    m = R.Model(_tiny_f32_model(1.0, 1.0, 128))
    logits = m.forward([0])
    assert logits.shape == (1, 100)


def test_generate_with_kv_cache_runs():  # forward.rs:786-839
    m = R.Model(_tiny_f32_model(0.0, 0.0, 32))
    kv = m.kv_cache(1, 32)
    out = m.generate([0, 1, 2], 5, kv)
    assert len(out) == 5 and all(t < 100 for t in out)
    assert len(kv) == 3 + 5
    # all logits are 0.0, and argmax keeps the last maximum (forward.rs:615-622)
    assert list(out) == [99] * 5


def test_decode_oov_token_is_invalid_index():  # forward.rs:552-554
    m = R.Model(_tiny_f32_model(0.0, 0.0, 32))
    kv = m.kv_cache(1, 32)
    with pytest.raises(R.OracleError) as e:
        m.decode_step(100, kv)
    assert e.value.name == "InvalidTensorIndex"
