"""The `ifx` program's inspect mode (src/main.rs:97-186) and argument
handling, on CPU: the output must equal, byte for byte, the text the
reference's print functions produce, restated below from main.rs and
value.rs (Display of values: integers, Rust's shortest round-trip float
text, booleans, strings, arrays previewed to eight items)."""
import math
import os
import struct
import subprocess
import sys

import numpy as np
import pytest

from gguf_builder import ARR, BOOL, F32V, F64, I8, I16, I32, I64, STR, U8, U16, U32, U64, GgufBuilder

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
IFX = os.path.join(ROOT, "inferox_b200", "ifx")
VT = ["uint8", "int8", "uint16", "int16", "uint32", "int32", "float32", "bool", "string", "array",
      "uint64", "int64", "float64"]
TT = {0: "F32", 1: "F16", 2: "Q4_0", 7: "Q8_0", 12: "Q4_K", 14: "Q6_K", 15: "Q8_K", 23: "IQ2_XXS"}
SIZES = {0: (1, 4), 1: (1, 2), 2: (32, 18), 7: (32, 34), 12: (256, 144), 14: (256, 210),
         15: (256, 292), 23: (256, 66)}
PACK = {U8: "<B", I8: "<b", U16: "<H", I16: "<h", U32: "<I", I32: "<i", F32V: "<f", BOOL: "<B",
        U64: "<Q", I64: "<q", F64: "<d"}


@pytest.fixture(scope="module", autouse=True)
def _built():
    if not os.path.exists(IFX):
        subprocess.run([sys.executable, os.path.join(ROOT, "inferox_b200", "build.py")], check=True)


def rust_float(v, single):
    if math.isnan(v):
        return "NaN"
    if math.isinf(v):
        return "inf" if v > 0 else "-inf"
    x = np.float32(v) if single else np.float64(v)
    s = np.format_float_positional(x, unique=True, trim="-")
    return "-0" if s == "-0" else s


def show(vt, v):
    if vt in (F32V, F64):
        return rust_float(v, vt == F32V)
    if vt == BOOL:
        return "true" if v else "false"
    if vt == STR:
        return v
    if vt == ARR:
        ety, items = v
        out = f"{VT[ety]}[{len(items)}] ["
        for i, it in enumerate(items):
            if i >= 8 and len(items) > 9:
                out += ", ..."
                break
            out += (", " if i else "") + show(ety, it)
        return out + "]"
    return str(v)


def payload(vt, v):
    if vt == STR:
        e = v.encode()
        return struct.pack("<Q", len(e)) + e
    if vt == ARR:
        ety, items = v
        return struct.pack("<IQ", ety, len(items)) + b"".join(payload(ety, it) for it in items)
    return struct.pack(PACK[vt], v)


def expected(path, meta, tensors, data_offset, file_len):
    rule = "-" * 72
    sec = lambda t: f"{rule}\n{t}\n{rule}\n"  # noqa: E731
    out = sec("Header") + f"  version:     3\n  n_tensors:   {len(tensors)}\n  n_kv:        {len(meta)}\n"
    out += sec(f"Metadata ({len(meta)} entries)")
    for i, (k, vt, v) in enumerate(meta):
        out += f"  [{i:3}] {k:50} ({VT[vt]}) => {show(vt, v)}\n"
    out += sec(f"Tensors ({len(tensors)} tensors)")
    total = 0
    for i, (name, shape, tt, off) in enumerate(tensors):
        n = int(np.prod(shape)) if shape else 1
        e, b = SIZES[tt]
        size = -(-n // e) * b
        total += size
        out += (f"  [{i:3}] {name}\n        type:    {TT[tt]} (id={tt})\n"
                f"        shape:   [{' x '.join(str(d) for d in shape)}]\n        elems:   {n}\n"
                f"        offset:  {off} bytes\n        size:    {size} bytes\n")
    out += sec("Layout") + (f"  file:                 {path}\n  tensor data offset:   {data_offset} bytes\n"
                            f"  total tensor bytes:   {total} bytes\n")
    out += sec("Raw tensor bytes (mmap)")
    if not tensors:
        out += "  (no tensors)\n"
    for name, shape, tt, off in tensors[:5]:
        n = int(np.prod(shape)) if shape else 1
        e, b = SIZES[tt]
        size = -(-n // e) * b
        if data_offset + off + size > file_len:
            out += f"  {name:40} -> error: unexpected end of file\n"
        else:
            out += f"  {name:40} -> {size} bytes\n"
    if len(tensors) > 5:
        out += f"  ... and {len(tensors) - 5} more tensor(s)\n"
    return out


def _write(tmp_path, meta, tensors, truncate=0):
    g = GgufBuilder()
    for k, vt, v in meta:
        g.raw_kv(k, vt, payload(vt, v))
    for name, shape, tt in tensors:
        n = int(np.prod(shape)) if shape else 1
        e, b = SIZES[tt]
        g.tensor(name, shape, tt, bytes((i * 7) & 255 for i in range(-(-n // e) * b)))
    raw = g.build()
    if truncate:
        raw = raw[:-truncate]
    p = tmp_path / "m.gguf"
    p.write_bytes(raw)
    return str(p), raw


def _offsets(tensors):
    offs, off = [], 0
    for _, shape, tt in tensors:
        offs.append(off)
        n = int(np.prod(shape)) if shape else 1
        e, b = SIZES[tt]
        off = (off + -(-n // e) * b + 31) // 32 * 32
    return offs


def _data_offset(raw, tensors):
    # the data region starts at the first 32-byte boundary after the infos
    return len(raw) - (_offsets(tensors)[-1] + _size(tensors[-1]) if tensors else 0) if tensors else None


def _size(t):
    _, shape, tt = t
    n = int(np.prod(shape)) if shape else 1
    e, b = SIZES[tt]
    return -(-n // e) * b


META = [
    ("general.architecture", STR, "llama"),
    ("u8", U8, 200), ("i8", I8, -5), ("u16", U16, 65000), ("i16", I16, -300),
    ("u32", U32, 4000000000), ("i32", I32, -7), ("u64", U64, 2 ** 63 + 5), ("i64", I64, -(2 ** 40)),
    ("eps", F32V, 1e-5), ("tenth", F32V, 0.1), ("big", F32V, 1e20), ("three", F32V, 3.0),
    ("negzero", F32V, -0.0), ("nan", F32V, float("nan")), ("inf", F32V, float("-inf")),
    ("pi64", F64, math.pi), ("tiny64", F64, 5e-324), ("flag", BOOL, 1), ("off", BOOL, 0),
    ("ключ.ünï", STR, "värde ✓"),
    ("arr.empty", ARR, (U32, [])), ("arr.three", ARR, (I32, [1, -2, 3])),
    ("arr.nine", ARR, (U8, list(range(9)))), ("arr.ten", ARR, (F32V, [0.5 * i for i in range(10)])),
    ("arr.strings", ARR, (STR, ["a", "b c", "", "☃"] * 4)),
    ("arr.nested", ARR, (ARR, [(U16, [1, 2]), (BOOL, [1, 0, 1])])),
]


def test_inspect_matches_reference_format(tmp_path):
    tensors = [("token_embd.weight", [256, 12], 12), ("output_norm.weight", [256], 0),
               ("blk.0.attn_v.weight", [256, 4], 14), ("a", [64], 7), ("b", [32, 2], 2),
               ("c", [33], 1), ("d", [512], 23)]
    path, raw = _write(tmp_path, META, tensors)
    offs = _offsets(tensors)
    data_offset = len(raw) - offs[-1] - _size(tensors[-1])
    r = subprocess.run([IFX, path], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    want = expected(path, META, [(n, s, t, o) for (n, s, t), o in zip(tensors, offs)], data_offset, len(raw))
    assert r.stdout == want


def test_inspect_truncated_and_empty(tmp_path):
    tensors = [("x", [256, 4], 12), ("y", [64], 0)]
    path, raw = _write(tmp_path, META[:3], tensors, truncate=100)
    offs = _offsets(tensors)
    data_offset = len(raw) + 100 - offs[-1] - _size(tensors[-1])
    r = subprocess.run([IFX, path], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    assert r.stdout == expected(path, META[:3], [(n, s, t, o) for (n, s, t), o in zip(tensors, offs)],
                                data_offset, len(raw))
    assert "y                                        -> error: unexpected end of file" in r.stdout
    path, raw = _write(tmp_path, [], [])
    r = subprocess.run([IFX, path], capture_output=True, text=True)
    assert r.returncode == 0 and "  (no tensors)\n" in r.stdout and "Metadata (0 entries)" in r.stdout


def test_errors_and_usage(tmp_path):
    r = subprocess.run([IFX], capture_output=True, text=True)
    assert r.returncode == 1 and r.stderr.startswith("usage: ")
    assert "<model.gguf> [tokenizer.json] [prompt] [max_tokens] [temperature]" in r.stderr
    bad = tmp_path / "bad.gguf"
    bad.write_bytes(b"GGML" + b"\0" * 40)
    r = subprocess.run([IFX, str(bad)], capture_output=True, text=True)
    assert r.returncode == 1
    assert r.stderr.strip() == f"error: failed to open '{bad}': invalid magic: expected 'GGUF', got [71, 71, 77, 76]"
    bad.write_bytes(b"GGUF" + struct.pack("<I", 7) + b"\0" * 40)
    r = subprocess.run([IFX, str(bad)], capture_output=True, text=True)
    assert r.returncode == 1 and "unsupported GGUF version: 7 (expected 2 or 3)" in r.stderr
    r = subprocess.run([IFX, str(tmp_path / "none.gguf")], capture_output=True, text=True)
    assert r.returncode == 1 and "io error: No such file or directory (os error 2)" in r.stderr
    # generate mode reports a tokenizer it cannot read before touching the model's data path
    path, _ = _write(tmp_path, META[:1], [])
    r = subprocess.run([IFX, path, str(tmp_path / "none.json"), "hi"], capture_output=True, text=True)
    assert r.returncode == 1 and r.stderr.startswith("error: failed to load ")


def test_kquant_layout_variable(tmp_path):
    path, _ = _write(tmp_path, META[:1], [])
    env = dict(os.environ, IFX_KQUANT_LAYOUT="gguf")
    r = subprocess.run([IFX, path, str(tmp_path / "t.json"), "hi"], capture_output=True, text=True, env=env)
    assert r.returncode == 1
    assert "IFX_KQUANT_LAYOUT must be 'reference' or 'ggml'" in r.stderr
