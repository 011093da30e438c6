"""The benchmark's workload definition exists twice: the product's generator
(inferox_b200.synth, which the GPU arm of bench.py uses) and the oracle's
(oracle/synth_ref.c, which the reference arm uses so that timing the
reference's CPU path never loads the product library). Both must produce the
same model, byte for byte, from the same table of shapes."""
import numpy as np
import pytest

from inferox_b200 import synth
from oracle import refcpu as R


def test_shape_tables_agree():
    assert R.BENCH_CONFIGS == synth.CONFIGS


@pytest.mark.parametrize("name,kw", [
    ("tiny", {}),
    (None, dict(vocab=2048, dim=512, n_layers=3, n_heads=8, n_kv_heads=2, ffn=1024, context=128,
                rope_base=500000.0, mix=1, tied=1, seed=99)),
    (None, dict(vocab=1024, dim=512, n_layers=2, n_heads=8, n_kv_heads=2, ffn=1024, mix=1, seed=3)),
    (None, dict(vocab=1024, dim=256, n_layers=2, n_heads=4, n_kv_heads=4, ffn=512, mix=2, seed=7)),
    ("1b", dict(n_layers=1, vocab=4096)),
])
def test_generators_agree_byte_for_byte(name, kw):
    a = R.synth_gguf(name, **kw)
    b = synth.build(name, **kw)
    assert a.size == b.size
    assert np.array_equal(a, b)
