"""The `ifx` program's generate mode (src/main.rs:39-95) on the GPU.

The prompt goes through the tokenizer and then token by token through
decode_step, the greedy tokens are decoded back to text, and stdout must
equal what the CPU oracle produces for the same steps (oracle tokenizer,
oracle decode_step loop, argmax, oracle decode). Sampling at a temperature
is reproducible under IFX_SEED; running past the model's context fails the
way main.rs does (exit 1, "error: decode failed: ...").
"""
import os
import subprocess
import sys

import pytest

from inferox_b200 import synth
from oracle import refcpu as R
from oracle import tokenizer_ref as T

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
IFX = os.path.join(ROOT, "inferox_b200", "ifx")
TOK = os.path.join(ROOT, "tests", "golden", "tokenizer_small.json")
R.set_threads(os.cpu_count() or 8)


@pytest.fixture(scope="module")
def model_path(tmp_path_factory):
    if not os.path.exists(IFX):
        subprocess.run([sys.executable, os.path.join(ROOT, "inferox_b200", "build.py")], check=True)
    g = synth.build(None, vocab=1024, dim=512, n_layers=2, n_heads=8, n_kv_heads=2, ffn=1024,
                    context=48, rope_base=500000.0, mix=1, seed=77)
    p = tmp_path_factory.mktemp("cli") / "small.gguf"
    p.write_bytes(g)
    return str(p), g


def _run(*args, env=None):
    e = dict(os.environ)
    e.update(env or {})
    return subprocess.run([IFX, *args], capture_output=True, env=e, timeout=300)


def test_generate_greedy_matches_oracle(model_path):
    path, g = model_path
    prompt = "klair tous, bézar ✓ <|im_start|>lou"
    tok = T.BpeTokenizer.from_json(open(TOK, encoding="utf-8").read())
    o = R.Model(g)
    kv = o.kv_cache(2, 48)
    logits = None
    for t in tok.encode(prompt):
        logits = o.decode_step(t, kv)
    out = []
    for _ in range(10):
        nxt = R.argmax(logits)
        out.append(nxt)
        logits = o.decode_step(nxt, kv)
    r = _run(path, TOK, prompt, "10")
    assert r.returncode == 0, r.stderr.decode()
    assert r.stdout.decode("utf-8") == tok.decode(out)
    # the default is 32 tokens at temperature 0; "+3" parses as 3
    assert _run(path, TOK, prompt, "+3").stdout == _run(path, TOK, prompt, "3", "0").stdout


def test_generate_sampled_reproducible_and_context_limit(model_path):
    path, _ = model_path
    a = _run(path, TOK, "tra sou", "12", "0.8", env={"IFX_SEED": "11"})
    b = _run(path, TOK, "tra sou", "12", "0.8", env={"IFX_SEED": "11"})
    assert a.returncode == 0 and a.stdout == b.stdout
    r = _run(path, TOK, "tra sou", "60")  # more steps than the 48-row context
    assert r.returncode == 1 and r.stderr.decode().startswith("error: decode failed: ")
