"""llama.cpp (ggml) byte orders on CPU: ifx_kquant_from_ggml, the block
permutation an IFX_KQUANT_GGML load applies, checked bit for bit.

For random blocks of each type, decoding llama.cpp's bytes with ggml's
formulas (oracle/ggml_ref.py) must equal decoding the converted bytes with
the reference's formulas (the oracle's dequantize, dequant.rs:62-199), with
Q6_K's scale bytes read as int8 (the only meaning change, which the kernels
take from the converted type). Also: the type-id mapping and the errors.
"""
import ctypes as C

import numpy as np
import pytest

from inferox_b200 import IfxError, _lib
from inferox_b200._lib import check
from oracle import ggml_ref as G
from oracle import refcpu as R


def convert(ggml_type: int, raw: bytes):
    out = (C.c_uint8 * max(1, len(raw)))()
    t, sgn = C.c_int(), C.c_int()
    check(_lib.lib.ifx_kquant_from_ggml(ggml_type, raw, len(raw), out, C.byref(t), C.byref(sgn)))
    return bytes(out)[: len(raw)], t.value, sgn.value


def ref_q6k_int8_scales(raw: bytes) -> np.ndarray:
    """dequant.rs:174-199 with the scale byte read as int8."""
    blk = np.frombuffer(raw, np.uint8).reshape(-1, 210)
    d = blk[:, 0:2].copy().view(np.float16).astype(np.float32)
    sc = blk[:, 2:18].view(np.int8).astype(np.float32)
    j = np.arange(256)
    ql = blk[:, 18 + j // 2].astype(np.int32)
    nib = np.where(j % 2 == 0, ql & 15, ql >> 4)
    hb = (blk[:, 146 + j // 4].astype(np.int32) >> (2 * (j % 4))) & 3
    q = nib | (hb << 4)
    return ((d * sc)[:, j // 16] * (q - 32).astype(np.float32)).astype(np.float32).reshape(-1)


def _random_blocks(ggml_type: int, nb: int, rng) -> bytes:
    e, n = G.BLOCK[ggml_type]
    b = rng.integers(0, 256, size=(nb, n), dtype=np.uint8)
    d = rng.uniform(-0.05, 0.05, size=(nb, 2)).astype(np.float16).view(np.uint8)
    if ggml_type == 14:
        b[:, 208:210] = d[:, 0:2]
    else:  # d (and Q4_K's dmin) lead the block
        b[:, 0:4] = d.reshape(nb, 4)[:, :4] if ggml_type == 12 else np.concatenate([d[:, :2], b[:, 2:4]], 1)
    return b.tobytes()


@pytest.mark.parametrize("name", ["Q4_0", "Q8_0", "Q4_K", "Q6_K"])
def test_conversion_decodes_identically(name):
    rng = np.random.default_rng(5)
    gt = G.GGML_IDS[name]
    raw = _random_blocks(gt, 64, rng)
    conv, t, sgn = convert(gt, raw)
    want = G.dequant(gt, raw)
    n = want.size
    if name == "Q6_K":
        assert (t, sgn) == (14, 1)
        got = ref_q6k_int8_scales(conv)
        # with every scale byte below 128 the reference's own reading agrees
        blk = np.frombuffer(conv, np.uint8).reshape(-1, 210).copy()
        blk[:, 2:18] &= 0x7F
        fixed = blk.tobytes()
        raw_fixed = np.frombuffer(raw, np.uint8).reshape(-1, 210).copy()
        raw_fixed[:, 192:208] &= 0x7F
        assert np.array_equal(R.dequantize(14, fixed, n).view(np.uint32),
                              G.dequant(14, raw_fixed.tobytes()).view(np.uint32))
    else:
        assert t == {"Q4_0": 2, "Q8_0": 7, "Q4_K": 12}[name] and sgn == 0
        got = R.dequantize(t, conv, n)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_in_place_conversion():
    rng = np.random.default_rng(11)
    for gt in (12, 14, 8):
        raw = _random_blocks(gt, 8, rng)
        want, _, _ = convert(gt, raw)
        buf = (C.c_uint8 * len(raw)).from_buffer_copy(raw)
        t, s = C.c_int(), C.c_int()
        check(_lib.lib.ifx_kquant_from_ggml(gt, buf, len(raw), buf, C.byref(t), C.byref(s)))
        assert bytes(buf) == want


def test_q4k_permutation_round_trip():
    rng = np.random.default_rng(9)
    ref = _random_blocks(12, 16, rng)
    back, t, _ = convert(12, G.q4k_reference_to_ggml(ref))
    assert t == 12 and back == ref


def test_q6k_quantiser_has_both_signs():
    rng = np.random.default_rng(3)
    x = rng.normal(0, 0.02, 256 * 8).astype(np.float32)
    raw = G.quantize_q6k_ggml(x, rng)
    sc = np.frombuffer(raw, np.uint8).reshape(-1, 210)[:, 192:208].view(np.int8)
    assert (sc < 0).any() and (sc > 0).any()
    y = G.dequant(14, raw)
    assert np.max(np.abs(y - x)) < 0.02 * 0.2  # a 6-bit quantiser's error


def test_type_ids_and_errors():
    out = (C.c_uint8 * 64)()
    t, s = C.c_int(), C.c_int()
    for ggml_id in (16, 30, 4):  # IQ2_XXS, BF16, removed id
        code = _lib.lib.ifx_kquant_from_ggml(ggml_id, bytes(64), 64, out, C.byref(t), C.byref(s))
        assert _lib.STATUS[code] == "Unsupported"
    code = _lib.lib.ifx_kquant_from_ggml(12, bytes(100), 100, out, C.byref(t), C.byref(s))
    assert _lib.STATUS[code] == "Shape"  # not whole 144-byte blocks
    with pytest.raises(IfxError):
        check(_lib.lib.ifx_kquant_from_ggml(12, None, 144, out, C.byref(t), C.byref(s)))
    raw = bytes(range(64))
    conv, tt, sg = convert(0, raw)  # F32: copied
    assert conv == raw and tt == 0 and sg == 0


@pytest.mark.parametrize("ggml_type", [2, 8, 12, 14])
def test_restatement_pinned_by_llama_cpp_gguf_py(ggml_type):
    """oracle/ggml_ref.py decodes llama.cpp's blocks exactly as llama.cpp's own
    Python package does (gguf-py 0.19.0, gguf.quants.dequantize, installed in
    this image): random block bytes with finite f16 scales, every type the
    ggml load path takes, bit for bit. Q6_K scale bytes take both signs."""
    gguf = pytest.importorskip("gguf")
    from gguf import quants

    elems, nbytes = G.BLOCK[ggml_type]
    nb = 400
    rng = np.random.default_rng(ggml_type)
    raw = rng.integers(0, 256, size=(nb, nbytes), dtype=np.uint8)
    scale_offsets = {2: [0], 8: [0], 12: [0, 2], 14: [208]}[ggml_type]
    for off in scale_offsets:
        raw[:, off:off + 2] = (rng.standard_normal(nb) * 0.01).astype(np.float16).view(np.uint8).reshape(nb, 2)
    raw = raw.reshape(-1)
    ours = G.dequant(ggml_type, raw)
    theirs = quants.dequantize(raw.reshape(nb, nbytes), gguf.GGMLQuantizationType(ggml_type))
    assert np.array_equal(ours, theirs.reshape(-1).astype(np.float32))
