"""CPU-only checks of the C ABI library: it loads without a GPU, exports every
entry point include/inferox.h declares, and its host-side pieces (synthetic
model generator, quantisers, GGUF writer) agree with the oracle."""
import ctypes as C
import os
import subprocess

import numpy as np
import pytest

import inferox_b200
from inferox_b200 import _lib, synth
from oracle import refcpu as R

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_library_exports_every_header_symbol():
    syms = inferox_b200.header_symbols()
    assert len(syms) >= 35
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    missing = [s for s in syms if s not in exported]
    assert not missing, missing


def test_status_names_mirror_gguf_error():
    # src/gguf/error.rs:6-42 in declaration order
    names = ["Io", "InvalidMagic", "UnsupportedVersion", "UnknownValueType", "UnknownTensorType",
             "InvalidUtf8", "InvalidShape", "UnexpectedEof", "TensorNotFound",
             "InvalidTensorIndex", "TensorOffsetOverflow", "UnsupportedArchitecture"]
    for i, n in enumerate(names, start=1):
        assert _lib.lib.ifx_status_name(i).decode() == n
        assert R.ERRORS[i] == n


def test_load_opts_defaults():
    o = inferox_b200.load_opts()
    assert o.tp_size == 1 and o.rope_compat == 1 and o.use_graphs == 1


@pytest.mark.parametrize("ttype,max_rel", [(2, 0.12), (7, 0.01), (12, 0.11), (14, 0.03)])
def test_quantisers_emit_reference_semantics(ttype, max_rel):
    x = synth.normal(11, 3, 0.02, 8192)
    y = R.dequantize(ttype, synth.quantize(ttype, x), x.size)
    rel = np.sqrt(np.mean((x - y) ** 2)) / np.sqrt(np.mean(x ** 2))
    assert rel < max_rel


def test_q6_k_scales_stay_below_128():
    # the reference reads Q6_K sub-scales as u8 (dequant.rs:184,195); the
    # quantiser keeps them in 0..127 so u8 and i8 readings agree
    x = synth.normal(5, 1, 0.02, 256 * 64)
    q = np.frombuffer(synth.quantize(14, x), np.uint8).reshape(-1, 210)
    assert q[:, 2:18].max() <= 127


def test_normal_generator_statistics():
    x = synth.normal(1234, 0, 0.02, 1 << 18)
    assert abs(x.mean()) < 2e-4
    assert abs(x.std() - 0.02) < 2e-4
    assert np.array_equal(x[:100], synth.normal(1234, 0, 0.02, 100))


@pytest.mark.parametrize("mix,tied", [(0, 0), (1, 0), (1, 1), (2, 0)])
def test_synth_gguf_parses_in_oracle(mix, tied):
    g = synth.build(None, vocab=512, dim=256, n_layers=2, n_heads=4, n_kv_heads=2, ffn=512,
                    context=64, mix=mix, tied=tied)
    m = R.Model(g)
    c = m.config
    assert (c.vocab_size, c.hidden_size, c.n_layers, c.n_heads, c.n_kv_heads) == (512, 256, 2, 4, 2)
    assert m.has_output() == (not tied)
    t_emb = m.tensor_info("token_embd.weight")[0]
    if mix == 1:
        assert m.tensor_info("blk.0.attn_v.weight")[0] == R.Q6_K
        assert m.tensor_info("blk.0.ffn_down.weight")[0] == R.Q6_K
        assert m.tensor_info("blk.1.ffn_down.weight")[0] == R.Q4_K
        assert m.tensor_info("blk.1.attn_q.weight")[0] == R.Q4_K
        assert t_emb == (R.Q6_K if tied else R.Q4_K)
    kv = m.kv_cache(2, 64)
    lg = m.decode_step(7, kv)
    assert np.isfinite(lg).all() and lg.std() > 0


def test_tiny_config_matches_baseline_shape():
    s = synth.spec("tiny")
    assert (s.dim, s.ffn, s.n_layers, s.n_heads, s.n_kv_heads, s.vocab) == (288, 768, 6, 6, 6, 32000)


def _load_status(data: bytes) -> str:
    h = C.c_void_p()
    buf = np.frombuffer(data, np.uint8)
    code = _lib.lib.ifx_model_load_mem(buf.ctypes.data_as(C.c_void_p), buf.nbytes, None, C.byref(h))
    assert not h.value
    return _lib.STATUS[code]


def test_model_load_rejects_bad_files_before_touching_a_gpu():
    # GgufFile::read / Config::from_gguf errors (file.rs:71-91, config.rs:35-42,
    # model/mod.rs:72-85) are host-side and carry the gguf::Error variant.
    import struct

    from gguf_builder import GgufBuilder, llama_meta
    assert _load_status(b"GGUX" + bytes(60)) == "InvalidMagic"
    assert _load_status(b"GGUF" + struct.pack("<IQQ", 9, 0, 0)) == "UnsupportedVersion"
    assert _load_status(b"GGUF" + struct.pack("<I", 3)) == "Io"
    g = GgufBuilder()
    g.string("general.architecture", "mamba")
    assert _load_status(g.build()) == "UnsupportedArchitecture"
    g = GgufBuilder()
    assert _load_status(g.build()) == "TensorNotFound"  # no general.architecture
    g = llama_meta(GgufBuilder(), 100, 64, 1, 4, 4, 128, 32)
    assert _load_status(g.build()) == "TensorNotFound"  # blk.0.* missing
    # zero kv heads: a Shape error, never an integer division by zero
    g = llama_meta(GgufBuilder(), 100, 64, 1, 4, 0, 128, 32)
    assert _load_status(g.build()) == "Shape"


def test_rust_binding_declares_every_entry_point():
    """The Rust extern block a maintainer copies into the reference crate
    (include/inferox_ffi.rs) declares every entry point of the header."""
    import re
    src = open(os.path.join(ROOT, "include", "inferox_ffi.rs")).read()
    declared = set(re.findall(r"pub fn (ifx_[a-z0-9_]+)", src))
    assert set(inferox_b200.header_symbols()) == declared


def test_plain_c_caller(tmp_path):
    """The header compiles as pedantic C99 and a C program links and runs."""
    exe = tmp_path / "c_caller"
    libdir = os.path.dirname(_lib.LIB_PATH)
    subprocess.run(["gcc", "-std=c99", "-Wall", "-Wextra", "-pedantic", "-Werror",
                    "-I", os.path.join(ROOT, "include"), os.path.join(ROOT, "tests", "cpp", "c_caller.c"),
                    "-L", libdir, "-linferox_b200", f"-Wl,-rpath,{libdir}", "-o", str(exe)], check=True)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0 and "c caller ok" in r.stdout, (r.returncode, r.stdout, r.stderr)
