"""RMSNorm producers (kernel-agent's rmsnorm_fp8 / rmsnorm_fp4 example producers,
src/kernel_agent/agent/examples/triton_fp8_producers.py:191-202 and
triton_fp4_producers.py:384-405) on the GPU, checked as the reference's own tests check them
(tests/test_fp8_toolkit.py, tests/test_fp4_producers.py): the codes and scales equal the
quantisation of the producer's own norm output bit for bit (the oracle's quantisers), and that
output equals eager RMSNorm (the oracle's) on at least 99 % of the elements. The FP4
producers' unbiased factor is outer times the oracle's fp4_bias_correction."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from helpers import np_bytes, np_values
from oracle import quant as oq

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(scope="module")
def prod():
    from kernel_agent_b200.kernels import producers

    return producers


def inputs(m, k, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    x = (torch.randn(m, k, generator=g) * 3).to(dtype)
    x[0, : k // 4] = 0.0
    w = (1.0 + 0.1 * torch.randn(k, generator=g)).to(dtype)
    return x.to(DEV), w.to(DEV)


def eager_share(out, x, w, dtype):
    ref = oq.rmsnorm(np_values(x), np_values(w), 1e-6, "bf16" if dtype == torch.bfloat16 else "f16")
    got = np_values(out)
    return float((got == ref).mean())


@pytest.mark.parametrize("m,k", [(353, 1024), (64, 4096), (5, 256), (130, 8192)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_rmsnorm_fp4_codes_of_its_output(prod, m, k, dtype):
    x, w = inputs(m, k, dtype, m + k)
    out = torch.empty(m, k, dtype=dtype, device=DEV)
    q, s, o, e = prod.rmsnorm_fp4(x, w, 1e-6, out=out, unbiased=True)
    h = np_values(out)
    rq, rs, ro = oq.quantize_fp4_activations(h)
    assert np.array_equal(np_bytes(q), rq) and np.array_equal(np_bytes(s), rs)
    assert np.array_equal(np_values(o), ro)
    want_e = (ro * oq.fp4_bias_correction(h, rq, rs, ro)).astype(np.float32)
    assert np.allclose(np_values(e), want_e, rtol=1e-6, atol=0)
    assert eager_share(out, x, w, dtype) >= 0.99
    # MXFP4 and swizzled scales from the same norm
    q2, s2, o2 = prod.rmsnorm_fp4(x, w, 1e-6, mx=True)
    rq2, rs2, ro2 = oq.quantize_fp4_activations(h, "mxfp4")
    assert np.array_equal(np_bytes(q2), rq2) and np.array_equal(np_bytes(s2), rs2)
    _, sw, _ = prod.rmsnorm_fp4(x, w, 1e-6, swizzle=True)
    assert np.array_equal(np_bytes(sw), oq.swizzle_scales(rs))


@pytest.mark.parametrize("m,k", [(353, 1024), (16, 4096), (3, 64)])
def test_rmsnorm_fp8_codes_of_its_output(prod, m, k):
    x, w = inputs(m, k, torch.bfloat16, 7 * m + k)
    out = torch.empty(m, k, dtype=torch.bfloat16, device=DEV)
    q, s = prod.rmsnorm_fp8(x, w, 1e-6, out=out)
    h = np_values(out)
    rq, rs = oq.quantize_fp8_activations(h)
    assert np.array_equal(np_bytes(q), rq) and np.array_equal(np_values(s), rs)
    assert eager_share(out, x, w, torch.bfloat16) >= 0.99
    if k % 32 == 0:
        qm, sm = prod.rmsnorm_fp8(x, w, 1e-6, mx=True)
        rqm, rsm = oq.quantize_mxfp8(h)
        assert np.array_equal(np_bytes(qm), rqm) and np.array_equal(np_bytes(sm), rsm)
        _, blocked = prod.rmsnorm_fp8(x, w, 1e-6, mx=True, blocked=True)
        assert np.array_equal(np_bytes(blocked), oq.swizzle_scales(rsm))


@pytest.mark.parametrize("m,k", [(300, 1024), (5, 2048), (7, 4096), (9, 8192), (33, 16384), (2, 32)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_rmsnorm_fp8_one_pass_equals_two(prod, m, k, dtype):
    """The fused producer (one pass over x: norm in registers, then the codes; for 2-byte rows
    128 or 256 threads with 1 to 8 chunks each across these widths) gives the bytes of the two
    passes (kab_rmsnorm into h, then the row / MXFP8 quantisers): h, codes and scales, per
    token and MXFP8 (row-major and swizzled); a row holding inf (r = 0, a NaN in h) included."""
    x, w = inputs(m, k, dtype, 5 * m + k)
    x[m - 1, 3] = float("inf")
    bits = torch.int32 if dtype == torch.float32 else torch.int16
    h1 = torch.empty(m, k, dtype=dtype, device=DEV)
    q1, s1 = prod.rmsnorm_fp8(x, w, 1e-5, out=h1)
    h2 = prod._rmsnorm(x, w, 1e-5, None)
    q2, s2 = prod.quantize_rows(h2)
    assert torch.equal(h1.view(bits), h2.view(bits))
    assert torch.equal(q1.view(torch.uint8), q2.view(torch.uint8)) and torch.equal(s1.view(torch.int32), s2.view(torch.int32))
    q3, s3 = prod.rmsnorm_fp8(x, w, 1e-5)  # h not written
    assert torch.equal(q3.view(torch.uint8), q2.view(torch.uint8))
    for blocked in (False, True):
        qm1, sm1 = prod.rmsnorm_fp8(x, w, 1e-5, mx=True, blocked=blocked)
        qm2, sm2 = prod.quantize_rows(h2, mx=True, blocked=blocked)
        assert torch.equal(qm1.view(torch.uint8), qm2.view(torch.uint8))
        assert torch.equal(sm1.view(torch.uint8), sm2.view(torch.uint8))


@pytest.mark.parametrize("m,k", [(300, 1024), (7, 4096), (5, 20480), (3, 32768), (2, 32)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_rmsnorm_fp4_one_pass_equals_two(prod, m, k, dtype):
    """The fused FP4 producer (kab_rmsnorm_quant_fp4: norm in registers, then the codes; 128 to
    512 threads and one to four blocks per thread across these widths) gives the bytes of the
    two passes (kab_rmsnorm into h, then kab_quant_fp4): h, codes, scales (row-major and
    swizzled) and outer scales, NVFP4 and MXFP4, with and without h written; a row holding
    inf (r = 0, NaN codes) included."""
    x, w = inputs(m, k, dtype, 3 * m + k)
    x[m - 1, 5] = float("inf")
    h2 = prod._rmsnorm(x, w, 1e-5, None)
    for mx in (False, True):
        for swizzle in (False, True):
            h1 = torch.empty(m, k, dtype=dtype, device=DEV)
            q1, s1, o1 = prod.rmsnorm_fp4(x, w, 1e-5, mx=mx, swizzle=swizzle, out=h1)
            q2, s2, o2 = prod.quantize_rows_fp4(h2, mx=mx, swizzle=swizzle)
            assert torch.equal(h1.view(torch.int16), h2.view(torch.int16))
            assert torch.equal(q1, q2) and torch.equal(s1.view(torch.uint8), s2.view(torch.uint8))
            assert torch.equal(o1.view(torch.int32), o2.view(torch.int32))
            q3, s3, o3 = prod.rmsnorm_fp4(x, w, 1e-5, mx=mx, swizzle=swizzle)  # h not written
            assert torch.equal(q3, q2) and torch.equal(s3.view(torch.uint8), s2.view(torch.uint8))
    _, _, o4, e4 = prod.rmsnorm_fp4(x, w, 1e-5, unbiased=True)  # h into a temporary
    _, _, _, e5 = prod.quantize_rows_fp4(h2, unbiased=True)
    assert torch.equal(e4.view(torch.int32), e5.view(torch.int32))


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_rmsnorm_fp4_wide_rows_on_a_second_device(prod):
    """Rows of 32768 elements need more than 48 KB of shared memory, a per-device function
    attribute: the first launch on the second GPU sets it there too (the first device's
    setting does not carry over)."""
    x0, w0 = inputs(3, 32768, torch.bfloat16, 11)
    prod.rmsnorm_fp4(x0, w0, 1e-5)  # device 0 first
    with torch.cuda.device(1):
        x, w = x0.to("cuda:1"), w0.to("cuda:1")
        q1, s1, o1 = prod.rmsnorm_fp4(x, w, 1e-5)
        q2, s2, o2 = prod.quantize_rows_fp4(prod._rmsnorm(x, w, 1e-5, None))
        assert torch.equal(q1, q2) and torch.equal(s1.view(torch.uint8), s2.view(torch.uint8))
        assert torch.equal(o1.view(torch.int32), o2.view(torch.int32))


def test_rmsnorm_fp4_fp32_takes_two_passes(prod):
    x, w = inputs(3, 1024, torch.float32, 13)
    out = torch.empty_like(x)
    q, s, o = prod.rmsnorm_fp4(x, w, 1e-6, out=out)
    rq, rs, ro = oq.quantize_fp4_activations(np_values(out))
    assert np.array_equal(np_bytes(q), rq) and np.array_equal(np_bytes(s), rs)
    assert np.array_equal(np_values(o), ro)


def test_rmsnorm_fp8_wide_rows_take_two_passes(prod):
    x, w = inputs(3, 16384 + 64, torch.bfloat16, 9)
    out = torch.empty_like(x)
    q, s = prod.rmsnorm_fp8(x, w, 1e-6, out=out)
    rq, rs = oq.quantize_fp8_activations(np_values(out))
    assert np.array_equal(np_bytes(q), rq) and np.array_equal(np_values(s), rs)


def test_unbiased_factor_of_the_other_fp4_producers(prod):
    x, _ = inputs(200, 2048, torch.bfloat16, 11)
    q, s, o, e = prod.quantize_rows_fp4(x, unbiased=True)
    h = np_values(x)
    rq, rs, ro = oq.quantize_fp4_activations(h)
    assert np.array_equal(np_bytes(q), rq) and np.array_equal(np_bytes(s), rs)
    assert np.allclose(np_values(e), ro * oq.fp4_bias_correction(h, rq, rs, ro), rtol=1e-6, atol=0)
    gu = (torch.randn(64, 2 * 1024, generator=torch.Generator().manual_seed(3)) * 2).to(torch.bfloat16).to(DEV)
    out = torch.empty(64, 1024, dtype=torch.bfloat16, device=DEV)
    q, s, o, e = prod.silu_mul_fp4(gu, out=out, unbiased=True)
    hv = np_values(out)
    rq, rs, ro = oq.quantize_fp4_activations(hv)
    assert np.array_equal(np_bytes(q), rq)
    assert np.allclose(np_values(e), ro * oq.fp4_bias_correction(hv, rq, rs, ro), rtol=1e-6, atol=0)
    q2, s2, o2, e2 = prod.silu_mul_fp4(gu, unbiased=True)  # the product into a temporary
    assert torch.equal(q2, q) and torch.equal(e2, e)


def test_rmsnorm_rejects_bad_shapes(prod):
    x = torch.randn(4, 100, device=DEV, dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        prod.rmsnorm_fp8(x, torch.ones(100, device=DEV, dtype=torch.bfloat16), 1e-6)
    x = torch.randn(4, 128, device=DEV, dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        prod.rmsnorm_fp4(x, torch.ones(64, device=DEV, dtype=torch.bfloat16), 1e-6)
