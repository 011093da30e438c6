"""ifx_op_sample_u_static: the sampler entry point whose scratch is a static
device array (it allocates nothing). Its picks must match ifx_op_sample_u's
on the same logits and draws, on two calls in a row (the second call reuses
the scratch the first one left behind).

This file is named to be collected last, so the entry point is also
exercised after every other GPU test has run in the same process.
"""
import ctypes as C

import numpy as np
import pytest
import torch
from cuda.bindings import driver as drv
from cuda.bindings import runtime as rt

from inferox_b200 import IfxError, ops
from inferox_b200._lib import SamplerC, check, lib

pytestmark = pytest.mark.gpu

LIMIT = 262144  # IFX_SAMPLE_STATIC_MAX


def _stream():
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


def sample_static(logits: torch.Tensor, temperature, top_k, top_p, u, out: torch.Tensor, slot: int):
    s = SamplerC(temperature, top_k, top_p)
    check(lib.ifx_op_sample_u_static(C.c_void_p(logits.data_ptr()), logits.numel(), C.byref(s),
                                     float(u), C.c_void_p(out[slot:].data_ptr()), _stream()),
          "sample_u_static")


SETTINGS = [
    (0.0, 0, 1.0),    # greedy: argmax, last index on ties
    (1.0, 0, 1.0),    # no truncation: candidates walked in index order
    (0.8, 40, 1.0),   # top-k
    (1.0, 0, 0.9),    # top-p
    (0.7, 50, 0.95),  # both
]


@pytest.mark.parametrize("n", [32000, 128256, LIMIT])
@pytest.mark.parametrize("temperature,top_k,top_p", SETTINGS)
def test_static_matches_allocating_sampler(n, temperature, top_k, top_p):
    rng = np.random.default_rng(n + int(temperature * 10) + top_k)
    logits = torch.from_numpy((rng.standard_normal(n) * 2).astype(np.float32)).to("cuda:0")
    out = torch.full((2,), -1, dtype=torch.int32, device="cuda:0")
    us = np.linspace(0.013, 0.987, 12)
    mism = [0, 0]
    for u in us:
        ref = ops.sample_u(logits, temperature, top_k, top_p, float(u))
        sample_static(logits, temperature, top_k, top_p, u, out, 0)
        sample_static(logits, temperature, top_k, top_p, u, out, 1)
        torch.cuda.synchronize()
        got = out.cpu().numpy().astype(np.int64)
        assert 0 <= got.min() and got.max() < n
        for k in range(2):
            mism[k] += int(got[k] != ref)
    # the same kernel over the same input: every mass sum is an exact integer
    # sum, so both calls pick exactly what the allocating entry point picks
    assert mism == [0, 0], mism


def _pool_high(pool) -> int:
    e, v = rt.cudaMemPoolGetAttribute(pool, rt.cudaMemPoolAttr.cudaMemPoolAttrUsedMemHigh)
    assert e == rt.cudaError_t.cudaSuccess
    return int(v)


def test_static_allocates_nothing():
    """Around a run of calls neither the device's free memory nor the default
    memory pool's high-water mark (reset first) moves."""
    n = 128256
    logits = torch.from_numpy(np.random.default_rng(1).standard_normal(n).astype(np.float32)).to("cuda:0")
    out = torch.zeros(4, dtype=torch.int32, device="cuda:0")
    # first calls on the device: the scratch address lookup, and lazy module
    # loading of each kernel the settings reach (driver memory for the code)
    for t, k, p in SETTINGS:
        sample_static(logits, t, k, p, 0.5, out, 0)
    torch.cuda.synchronize()
    e, pool = rt.cudaDeviceGetDefaultMemPool(0)
    assert e == rt.cudaError_t.cudaSuccess
    (e,) = rt.cudaMemPoolSetAttribute(pool, rt.cudaMemPoolAttr.cudaMemPoolAttrUsedMemHigh,
                                     drv.cuuint64_t(0))
    assert e == rt.cudaError_t.cudaSuccess
    high0 = _pool_high(pool)
    free0, _ = torch.cuda.mem_get_info(0)
    for i, (t, k, p) in enumerate(SETTINGS * 4):
        sample_static(logits, t, k, p, (i + 0.5) / 20, out, i % 4)
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info(0)
    assert free1 == free0
    assert _pool_high(pool) == high0


def test_static_rejects_beyond_limit():
    logits = torch.zeros(LIMIT + 1, dtype=torch.float32, device="cuda:0")
    out = torch.zeros(1, dtype=torch.int32, device="cuda:0")
    with pytest.raises(IfxError) as e:
        sample_static(logits, 1.0, 0, 1.0, 0.5, out, 0)
    assert e.value.name == "InvalidArgument"
    assert str(LIMIT) in str(e.value)
    s = SamplerC(1.0, 0, 1.0)
    with pytest.raises(IfxError) as e:  # empty logits (a valid pointer, n = 0)
        check(lib.ifx_op_sample_u_static(C.c_void_p(logits.data_ptr()), 0, C.byref(s), 0.5,
                                         C.c_void_p(out.data_ptr()), _stream()), "sample_u_static")
    assert e.value.name == "Shape"
