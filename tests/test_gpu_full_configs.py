"""Parity at the full shapes the benchmark times, on the benchmark's own inputs.

The GEMM tile schedule depends on the shape: with N > M the n-panels sweep m, and N = 28672 =
149 x 192 + 64 leaves a ragged last panel. So config 4 (X [8192, 8192] x W [28672, 8192]^T,
NVFP4) and config 3 (SiLU(gate) * up -> MXFP8, then the [4096, 14336] x [4096, 14336]^T
down-projection) are checked here at those shapes: spread rows across every output column
against the oracle's float64 dequant-matmul of the same codes, at the north-star tolerance
(bf16 atol / rtol 2e-2 with at most 0.1 % outside, relative L2 <= 0.02, cosine >= 0.999, and
>= 99 % of outputs within one bf16 step). The comparator's verdict on a config-4-sized output
pair is checked against the oracle over all 235 M elements."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from helpers import np_bf16_bits, np_bytes, np_values, ulp_distance_bf16
from oracle import compare as ocmp
from oracle import quant as oq
from oracle.formats import f32_to_bf16

pytestmark = pytest.mark.gpu
DEV = "cuda"
# tile edges (128-row m-tiles), both ends and a few rows in between
ROWS_8192 = [0, 1, 127, 128, 129, 255, 256, 1023, 1024, 2047, 4095, 4096, 6143, 8063, 8064, 8191]
ROWS_4096 = [0, 1, 127, 128, 255, 256, 1023, 1024, 2047, 2048, 3071, 3967, 3968, 4094, 4095]


def check_close(got_bits: np.ndarray, want: np.ndarray, label: str) -> None:
    """The north-star tolerance of a bf16 output against fp32 oracle values."""
    got = np.ascontiguousarray(got_bits, np.uint16).view(np.uint16).astype(np.uint32) << 16
    got = got.view(np.float32).astype(np.float64)
    ref = want.astype(np.float64)
    diff = np.abs(got - ref)
    mism = float((diff > 2e-2 + 2e-2 * np.abs(ref)).mean())
    rel = float(np.linalg.norm(got - ref) / max(np.linalg.norm(ref), 1e-30))
    cos = float((got.ravel() @ ref.ravel()) / max(np.linalg.norm(got) * np.linalg.norm(ref), 1e-30))
    ulps = ulp_distance_bf16(got_bits.reshape(-1), f32_to_bf16(want).reshape(-1))
    msg = f"{label}: mismatch {mism:.2e} rel_l2 {rel:.3e} cos {cos:.7f} within 1 ulp {np.mean(ulps <= 1):.4f}"
    assert mism <= 1e-3 and rel <= 0.02 and cos >= 0.999, msg
    assert float(np.mean(ulps <= 1)) >= 0.99, msg


def test_config4_w4a4_linear_at_the_benchmark_shape():
    """fp4_w4a4_linear at M = 8192, K = 8192, N = 28672 (seed 0, the benchmark's inputs):
    16 spread rows x all 28672 columns against the oracle, the ragged last 64-column panel
    (28608-28671) on its own, and a second call bit-identical."""
    from kernel_agent_b200 import workloads
    from kernel_agent_b200.kernels import quant

    x, w, b = workloads.config4(seed=0, device="cuda")
    m, k = x.shape
    n = w.shape[0]
    assert (m, k, n) == (8192, 8192, 28672)
    q, s, ts = quant.quantize_fp4(w)
    del w
    y = quant.fp4_w4a4_linear(x, q, s, ts, b)
    assert y.shape == (m, n) and y.dtype == torch.bfloat16
    got = np_bf16_bits(y[ROWS_8192])
    xr, bias = np_values(x[ROWS_8192]), np_values(b)
    codes, scales = np_bytes(q), np_bytes(s)
    want = np.empty((len(ROWS_8192), n), np.float32)
    step = 4096  # oracle column chunks: the float64 weight values of a chunk are 268 MB
    for c0 in range(0, n, step):
        cols = slice(c0, min(n, c0 + step))
        want[:, cols] = oq.fp4_w4a4_linear(xr, codes[cols], scales[cols], float(ts), bias[cols], out_dtype="f32")
    check_close(got, want, "config 4, all columns")
    check_close(got[:, 28608:], want[:, 28608:], "config 4, ragged last panel")
    y2 = quant.fp4_w4a4_linear(x, q, s, ts, b)
    assert torch.equal(y, y2)


def test_config3_mlp_down_projection_at_the_benchmark_shape():
    """Config 3's MLP block at its shape: the fused SiLU(gate) * up -> MXFP8 producer on
    gate, up [4096, 14336], then the down-projection GEMM against W_down [4096, 14336]
    (kind::mxf8f6f4, e8m0 per 32 on both operands). The producer's codes of 15 spread rows
    are the oracle's quantisation of the producer's own product; the GEMM's rows over all
    4096 columns are the oracle's float64 matmul of the same codes."""
    from kernel_agent_b200 import workloads
    from kernel_agent_b200.kernels import gemm, producers, quant

    gate, up, wd = workloads.config3(seed=0, device="cuda")
    m, f = gate.shape
    hdim = wd.shape[0]
    assert (m, f, hdim) == (4096, 14336, 4096)
    wq, ws = quant.quantize_mxfp8(wd)
    del wd
    h = torch.empty_like(gate)
    xq, xs = producers.silu_mul_fp8(gate, up, mx=True, blocked=False, out=h)
    xq_b, xs_b = producers.silu_mul_fp8(gate, up, mx=True, blocked=True)
    assert torch.equal(xq.view(torch.uint8), xq_b.view(torch.uint8))
    # the codes are the oracle's MXFP8 quantisation of the producer's own SiLU * up product
    rq, rs = oq.quantize_mxfp8(np_values(h[ROWS_4096]))
    assert np.array_equal(np_bytes(xq[ROWS_4096]), rq)
    assert np.array_equal(np_bytes(xs[ROWS_4096]), rs)
    # the products are >= 99 % bit-equal to eager SiLU * up (the reference tests' contract)
    eager = torch.nn.functional.silu(gate[ROWS_4096]) * up[ROWS_4096]
    assert float((eager.view(torch.int16) == h[ROWS_4096].view(torch.int16)).float().mean()) >= 0.99
    y = gemm.mxf8(xq_b, xs_b, wq, quant.swizzle_mx_scales(ws).view(torch.uint8), None, out_dtype=torch.bfloat16)
    assert y.shape == (m, hdim)
    want = oq.mxfp8_linear_codes(np_bytes(xq[ROWS_4096]), np_bytes(xs[ROWS_4096]), np_bytes(wq), np_bytes(ws),
                                 None, out_dtype="f32")
    check_close(np_bf16_bits(y[ROWS_4096]), want, "config 3 down-projection")


def test_comparator_verdict_on_a_config4_sized_pair():
    """The benchmark's comparator pair (bf16 [8192, 28672], new = ref x (1 + 0.01 N(0, 1))):
    the exact tier's verdict, mismatch fraction and worst ratio equal the oracle's over all
    235 M elements (the kernel's 32-bit chunk counts and float partial sums must not lose
    them); cosine and relative L2 within the reference's fp32 reduction noise."""
    from kernel_agent_b200.kernels import compare

    g = torch.Generator(device=DEV).manual_seed(0)
    shape = (8192, 28672)
    ref = torch.randn(*shape, generator=g, device=DEV).to(torch.bfloat16)
    new = (ref.float() * (1 + 0.01 * torch.randn(*shape, generator=g, device=DEV))).to(torch.bfloat16)
    got = compare.compare_tensors("y", ref, new)
    want = ocmp.compare_tensors("y", np_values(ref), np_values(new), "bf16")
    assert got["ok"] == want["ok"], (got, want)
    for key in ("mismatch_frac", "max_err_ratio", "max_abs_err"):
        assert got[key] == want[key], (key, got[key], want[key])
    assert abs(got["cosine"] - want["cosine"]) <= 2e-5 and abs(got["rel_l2"] - want["rel_l2"]) <= 2e-4 * want["rel_l2"]
    assert ("error" in got) == ("error" in want)
