"""numpy restatement of llama.cpp's (ggml's) quantised block formats (test
infrastructure: the checker for the IFX_KQUANT_GGML load path, never on the
product path).

The reference decodes only its own byte orders (src/gguf/dequant.rs:62-232)
and numbers tensor types its own way (src/gguf/types.rs:70-100); llama.cpp
is not part of the reference and not vendored anywhere here, so these
functions restate ggml's published block formats (ggml-quants.c's
dequantize_row_q4_0 / q8_0 / q4_K / q6_K and the block structs of
ggml-common.h) from their definitions:

  Q4_0  {f16 d; u8 qs[16]}          y[j] = (nibble - 8) * d, low nibbles first
  Q8_0  {f16 d; i8 qs[32]}          y[j] = qs[j] * d
  Q4_K  {f16 d, dmin; u8 scales[12]; u8 qs[128]}
        64-element chunk c: elements 64c..64c+31 are the low nibbles of
        qs[32c..32c+31] with scale/min 2c, the next 32 the high nibbles with
        2c+1; 6-bit scale/min unpacking as in the reference (dequant.rs:141-149);
        y = (d * sc) * q - (dmin * m)
  Q6_K  {u8 ql[128]; u8 qh[64]; i8 scales[16]; f16 d}
        element 128n + 32t + l: low (t < 2) or high (t >= 2) nibble of
        ql[64n + 32(t & 1) + l], bits 2t..2t+1 of qh[32n + l] as bits 4-5;
        y = (d * scales[j / 16]) * (q - 32)

Every product is rounded to f32 separately (numpy float32 arithmetic); a
llama.cpp build that contracts these into FMAs may differ in the last bit,
which is why the model-level check is the logits tolerance.
"""
from __future__ import annotations

import numpy as np

GGML_IDS = {"F32": 0, "F16": 1, "Q4_0": 2, "Q8_0": 8, "Q4_K": 12, "Q6_K": 14}
BLOCK = {0: (1, 4), 1: (1, 2), 2: (32, 18), 8: (32, 34), 12: (256, 144), 14: (256, 210)}


def _f16(b: np.ndarray) -> np.ndarray:
    return b.copy().view(np.float16).astype(np.float32).reshape(-1)


def _scale_min_k4(sc: np.ndarray):
    """[nb, 12] bytes -> ([nb, 8] scales, [nb, 8] mins), dequant.rs:141-149."""
    sc = sc.astype(np.uint32)
    s = np.zeros((sc.shape[0], 8), np.uint32)
    m = np.zeros_like(s)
    for g in range(8):
        if g < 4:
            s[:, g] = sc[:, g] & 63
            m[:, g] = sc[:, g + 4] & 63
        else:
            s[:, g] = (sc[:, g + 4] & 15) | ((sc[:, g - 4] >> 6) << 4)
            m[:, g] = (sc[:, g + 4] >> 4) | ((sc[:, g] >> 6) << 4)
    return s.astype(np.float32), m.astype(np.float32)


def dequant(ggml_type: int, raw: bytes | np.ndarray) -> np.ndarray:
    b = np.frombuffer(bytes(raw), np.uint8)
    if ggml_type == 0:
        return b.view(np.float32).copy()
    if ggml_type == 1:
        return b.view(np.float16).astype(np.float32)
    e, n = BLOCK[ggml_type]
    blk = b.reshape(-1, n)
    nb = blk.shape[0]
    if ggml_type == 2:
        d = _f16(blk[:, 0:2])[:, None]
        qs = blk[:, 2:18].astype(np.int32)
        q = np.concatenate([qs & 15, qs >> 4], axis=1) - 8
        return (q.astype(np.float32) * d).reshape(-1)
    if ggml_type == 8:
        d = _f16(blk[:, 0:2])[:, None]
        return (blk[:, 2:34].view(np.int8).astype(np.float32) * d).reshape(-1)
    if ggml_type == 12:
        d = _f16(blk[:, 0:2])[:, None]
        dmin = _f16(blk[:, 2:4])[:, None]
        s, m = _scale_min_k4(blk[:, 4:16])
        qs = blk[:, 16:144].reshape(nb, 4, 32).astype(np.uint32)
        q = np.stack([qs & 15, qs >> 4], axis=2).reshape(nb, 256).astype(np.float32)  # [c][lo/hi][l]
        sc = np.repeat(d * s, 32, axis=1)
        mn = np.repeat(dmin * m, 32, axis=1)
        return (sc * q - mn).astype(np.float32).reshape(-1)
    if ggml_type == 14:
        ql = blk[:, 0:128].astype(np.uint32)
        qh = blk[:, 128:192].astype(np.uint32)
        sc = blk[:, 192:208].view(np.int8).astype(np.float32)
        d = _f16(blk[:, 208:210])[:, None]
        q = np.zeros((nb, 256), np.int32)
        for j in range(256):
            n_, t, l = j // 128, (j % 128) // 32, j % 32
            byte = ql[:, 64 * n_ + 32 * (t & 1) + l]
            lo = (byte & 15) if t < 2 else (byte >> 4)
            hi = (qh[:, 32 * n_ + l] >> (2 * t)) & 3
            q[:, j] = (lo | (hi << 4)).astype(np.int32)
        ds = d * sc  # [nb, 16]
        return (np.repeat(ds, 16, axis=1) * (q - 32).astype(np.float32)).astype(np.float32).reshape(-1)
    raise ValueError(f"ggml type {ggml_type}")


def q4k_reference_to_ggml(raw: bytes) -> bytes:
    """Reference-order Q4_K blocks (dequant.rs:123-163) rewritten in ggml's
    order (for building llama.cpp-style test files)."""
    blk = np.frombuffer(raw, np.uint8).reshape(-1, 144)
    out = blk.copy()
    nb = blk.shape[0]
    qs = blk[:, 16:].astype(np.uint8)
    vals = np.zeros((nb, 256), np.uint8)  # reference: byte 16g + l/2, even l low
    for j in range(256):
        g, l = j // 32, j % 32
        byte = qs[:, 16 * g + l // 2]
        vals[:, j] = (byte & 15) if l % 2 == 0 else (byte >> 4)
    new = np.zeros((nb, 128), np.uint8)
    for c in range(4):
        new[:, 32 * c:32 * c + 32] = vals[:, 64 * c:64 * c + 32] | (vals[:, 64 * c + 32:64 * c + 64] << 4)
    out[:, 16:] = new
    return out.tobytes()


def quantize_q6k_ggml(x: np.ndarray, rng: np.random.Generator) -> bytes:
    """A Q6_K quantiser in ggml's layout whose int8 scales take both signs
    (llama.cpp's own quantiser produces negative scales; here the sign of
    each 16-element group's scale is random and q absorbs it)."""
    x = np.asarray(x, np.float32).reshape(-1, 256)
    nb = x.shape[0]
    out = np.zeros((nb, 210), np.uint8)
    g = x.reshape(nb, 16, 16)
    amax = np.abs(g).max(axis=2)  # [nb, 16]
    bmax = np.maximum(amax.max(axis=1), 1e-12)  # [nb]
    d = (bmax / (127.0 * 31.0)).astype(np.float16)
    d32 = np.maximum(d.astype(np.float32), np.float32(6e-8))
    sign = np.where(rng.random((nb, 16)) < 0.5, -1, 1)
    sc = np.clip(np.round(amax / (d32[:, None] * 31.0)), 1, 127).astype(np.int32) * sign
    step = d32[:, None] * sc.astype(np.float32)  # [nb, 16]
    q = np.clip(np.round(g / step[:, :, None]), -32, 31).astype(np.int32) + 32  # [nb,16,16]
    q = q.reshape(nb, 256)
    ql = np.zeros((nb, 128), np.uint8)
    qh = np.zeros((nb, 64), np.uint8)
    for j in range(256):
        n_, t, l = j // 128, (j % 128) // 32, j % 32
        lo, hi = q[:, j] & 15, (q[:, j] >> 4) & 3
        ql[:, 64 * n_ + 32 * (t & 1) + l] |= (lo if t < 2 else lo << 4).astype(np.uint8)
        qh[:, 32 * n_ + l] |= (hi << (2 * t)).astype(np.uint8)
    out[:, 0:128] = ql
    out[:, 128:192] = qh
    out[:, 192:208] = sc.astype(np.int8).view(np.uint8)
    out[:, 208:210] = d.reshape(nb, 1).view(np.uint8)
    return out.tobytes()
