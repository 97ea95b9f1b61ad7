"""The CPU execution path the benchmark times (``oracle/cpu_path.py``, the reference's fp32
CPU arithmetic) agrees with the oracle's exact restatements: integer products bit for bit,
fp32-accumulated results within the comparator's bf16 tolerance of the float64 ones."""

from __future__ import annotations

import numpy as np
import torch

from oracle import cpu_path, fp8lib
from oracle import quant as oq
from oracle.formats import bf16_to_f32


def bf16(t: torch.Tensor) -> np.ndarray:
    return bf16_to_f32(t.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16))


def close(got_bits, want_f32, tol=2e-2):
    got = bf16_to_f32(got_bits).astype(np.float64)
    want = np.asarray(want_f32, np.float64)
    assert np.mean(np.abs(got - want) > tol + tol * np.abs(want)) <= 1e-3
    assert np.linalg.norm(got - want) <= 0.01 * np.linalg.norm(want)


def test_int8_path_is_exact():
    g = torch.Generator().manual_seed(0)
    a = torch.randint(-127, 128, (33, 2304), generator=g, dtype=torch.int8).numpy()
    b = torch.randint(-127, 128, (40, 2304), generator=g, dtype=torch.int8).numpy()
    assert np.array_equal(cpu_path.int8_matmul(a, b), oq.int8_matmul(a, b))
    x = bf16(torch.randn(16, 1024, generator=g))
    q, s = oq.quantize_int8(bf16(torch.randn(64, 1024, generator=g) * 0.02))
    assert np.array_equal(cpu_path.int8_w8a8_linear(x, q, s), oq.int8_w8a8_linear(x, q, s))


def test_fp4_mxfp8_blockwise_and_attention_paths():
    g = torch.Generator().manual_seed(1)
    x = bf16(torch.randn(24, 512, generator=g))
    w = bf16(torch.randn(96, 512, generator=g) * 0.01)
    codes, scales, ts = oq.quantize_fp4(w)
    b = bf16(torch.randn(96, generator=g) * 0.05)
    close(cpu_path.fp4_w4a4_linear(x, codes, scales, ts, b), oq.fp4_w4a4_linear(x, codes, scales, ts, b, out_dtype="f32"))
    # a slice of the weight's rows quantised with the whole weight's amax: the slice of the codes
    c2, s2, t2 = oq.quantize_fp4(w[:40], amax=float(np.abs(w).max()))
    assert np.array_equal(c2, codes[:40]) and np.array_equal(s2, scales[:40]) and t2 == ts
    xq, xs = oq.quantize_mxfp8(x)
    wq, ws = oq.quantize_mxfp8(w)
    close(cpu_path.mxfp8_linear_codes(xq, xs, wq, ws), oq.mxfp8_linear_codes(xq, xs, wq, ws, out_dtype="f32"))
    gq, gs = cpu_path.silu_mul_mxfp8(x, x[::-1])
    rq, rs = oq.quantize_mxfp8(oq.silu_mul(x, x[::-1]))
    assert np.array_equal(gq, rq) and np.array_equal(gs, rs)
    w3 = bf16(torch.randn(256, 512, generator=g) * 0.02)
    bq, bs = fp8lib.quantize_fp8_blocks(w3)
    want = fp8lib.fp8_blockwise_gemm(*fp8lib.quantize_fp8_groups(x), bq, bs, out_dtype="f32")
    close(cpu_path.fp8_blockwise_linear(x, bq, bs), want)
    q, k, v = (bf16(torch.randn(64, 128, generator=g)) for _ in range(3))
    a = cpu_path.attention_fp8_head(q, k, v)
    ref = fp8lib.attention_fp8_head(q, k, v)
    assert np.linalg.norm(a - ref) <= 1e-3 * np.linalg.norm(ref)
