"""The tcgen05 scaled GEMMs against the oracle: int8 products and the W8A8 INT8 linear bit
for bit; FP8 / MXFP8 / NVFP4 linears within the bf16 tolerances the comparator applies
(atol = rtol = 2e-2, relative L2 <= 0.02, cosine >= 0.999) and, tighter, within one bf16
step of the float64-accumulated oracle on >= 99 % of the outputs."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from helpers import np_bf16_bits, np_bytes, np_values, ulp_distance_bf16
from oracle import quant as oq
from oracle.formats import bf16_to_f32, f32_to_bf16

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(scope="module")
def kq():
    from kernel_agent_b200.kernels import quant

    return quant


def rand_i8(g, *shape):
    return torch.randint(-127, 128, shape, generator=g, dtype=torch.int8)


def diagnose(got: np.ndarray, want: np.ndarray) -> str:
    """A short description of how an integer product differs (layout bugs show as patterns)."""
    bad = got != want
    lines = [f"mismatch {bad.mean():.4f} of {bad.size}"]
    idx = np.argwhere(bad)[:6]
    for i, j in idx:
        lines.append(f"  [{i},{j}] got {got[i, j]} want {want[i, j]}")
    # which reference row / column does each output row / column equal?
    for i in range(min(4, got.shape[0])):
        hits = [r for r in range(want.shape[0]) if np.array_equal(got[i], want[r])]
        lines.append(f"  row {i} equals reference rows {hits[:4]}")
    for j in range(min(4, got.shape[1])):
        hits = [c for c in range(want.shape[1]) if np.array_equal(got[:, j], want[:, c])]
        lines.append(f"  col {j} equals reference cols {hits[:4]}")
    lines.append(f"  got[0,:8] {got[0, :8].tolist()}")
    lines.append(f"  want[0,:8] {want[0, :8].tolist()}")
    return "\n".join(lines)


def close_bf16(y: torch.Tensor, want_f32: np.ndarray, label: str) -> None:
    got = np_values(y).astype(np.float64)
    ref = want_f32.astype(np.float64)
    diff = np.abs(got - ref)
    allowed = 2e-2 + 2e-2 * np.abs(ref)
    mism = float((diff > allowed).mean())
    rel = float(np.linalg.norm(got - ref) / max(np.linalg.norm(ref), 1e-30))
    cos = float((got.ravel() @ ref.ravel()) / max(np.linalg.norm(got) * np.linalg.norm(ref), 1e-30))
    ulps = ulp_distance_bf16(np_bf16_bits(y).reshape(-1), f32_to_bf16(want_f32).reshape(-1))
    msg = f"{label}: mismatch {mism:.2e} rel_l2 {rel:.3e} cos {cos:.7f} same {np.mean(ulps == 0):.4f} max ulps {ulps.max()}"
    assert mism <= 1e-3 and rel <= 0.02 and cos >= 0.999, msg
    assert float(np.mean(ulps <= 1)) >= 0.99, msg


def close_bf16_tol(y: torch.Tensor, want_f32: np.ndarray, label: str) -> None:
    """The comparator's exact-tier bf16 checks (atol = rtol = 2e-2, <= 0.1 % outside, relative
    L2 <= 0.02, cosine >= 0.999)."""
    got = np_values(y).astype(np.float64)
    ref = want_f32.astype(np.float64)
    mism = float((np.abs(got - ref) > 2e-2 + 2e-2 * np.abs(ref)).mean())
    rel = float(np.linalg.norm(got - ref) / max(np.linalg.norm(ref), 1e-30))
    cos = float((got.ravel() @ ref.ravel()) / max(np.linalg.norm(got) * np.linalg.norm(ref), 1e-30))
    assert mism <= 1e-3 and rel <= 0.02 and cos >= 0.999, (label, mism, rel, cos)


def test_int8_products_layout():
    g = torch.Generator().manual_seed(0)
    a = rand_i8(g, 128, 128)
    b = rand_i8(g, 256, 128)
    from kernel_agent_b200.kernels import quant

    got = quant.int8_matmul(a.to(DEV), b.to(DEV)).cpu().numpy()
    want = oq.int8_matmul(a.numpy(), b.numpy())
    assert np.array_equal(got, want), diagnose(got, want)


@pytest.mark.parametrize("m,k,n", [(1, 128, 8), (5, 3000, 24), (17, 4096, 40), (128, 1024, 1024),
                                   (300, 512, 520), (1000, 256, 4096), (2, 4096, 3)])
def test_int8_matmul_exact(kq, m, k, n):
    g = torch.Generator().manual_seed(m * 7 + n)
    a, b = rand_i8(g, m, k), rand_i8(g, n, k)
    got = kq.int8_matmul(a.to(DEV), b.to(DEV))
    assert got.dtype == torch.int32 and tuple(got.shape) == (m, n)
    want = oq.int8_matmul(a.numpy(), b.numpy())
    g2 = got.cpu().numpy()
    assert np.array_equal(g2, want), diagnose(g2, want)
    worst = torch.full((2, 4096), 127, dtype=torch.int8, device=DEV)
    assert int(kq.int8_matmul(worst, -worst)[0, 0]) == -4096 * 127 * 127


def test_int8_w8a8_linear_bit_exact_config1_and_golden(kq, golden):
    from kernel_agent_b200 import workloads

    x, w, b = workloads.config1(seed=0)
    q, s = kq.quantize_int8(w.to(DEV))
    y = kq.int8_w8a8_linear(x.to(DEV), q, s, b.to(DEV))
    want = oq.int8_w8a8_linear(np_values(x), np_bytes(q).view(np.int8), s.cpu().numpy(), np_values(b))
    assert y.dtype == torch.bfloat16 and np.array_equal(np_bf16_bits(y), want)
    g = golden
    xg = torch.from_numpy(g["int8_x"].view(np.int16)).view(torch.bfloat16).to(DEV)
    wq = torch.from_numpy(g["int8_wq"]).to(DEV)
    ws = torch.from_numpy(g["int8_ws"]).to(DEV)
    bg = torch.from_numpy(g["int8_bias"].view(np.int16)).view(torch.bfloat16).to(DEV)
    y = kq.int8_w8a8_linear(xg, wq, ws, bg)
    assert np.array_equal(np_bf16_bits(y), g["int8_y"])  # the reference's own output bits
    # [..., K] inputs keep their leading shape; fp32 activations give fp32 outputs
    x3 = torch.randn(3, 7, 1024, generator=torch.Generator().manual_seed(1))
    y3 = kq.int8_w8a8_linear(x3.to(DEV), q, s)
    want3 = oq.int8_w8a8_linear(x3.numpy(), np_bytes(q).view(np.int8), s.cpu().numpy(), None, out_dtype="f32")
    assert y3.shape == (3, 7, 1024) and np.array_equal(y3.reshape(21, -1).cpu().numpy(), want3)


@pytest.mark.parametrize("m,k,n", [(128, 1024, 1024), (33, 512, 384), (2048, 1024, 3072)])
def test_fp8_w8a8_linear(kq, m, k, n):
    g = torch.Generator().manual_seed(m + k)
    x = torch.randn(m, k, generator=g).to(torch.bfloat16)
    w = (torch.randn(n, k, generator=g) * 0.02).to(torch.bfloat16)
    b = (torch.randn(n, generator=g) * 0.1).to(torch.bfloat16)
    q, s = kq.quantize_fp8(w.to(DEV))
    y = kq.fp8_w8a8_linear(x.to(DEV), q, s, b.to(DEV))
    xq, xs = oq.quantize_fp8_activations(np_values(x))
    from oracle.formats import e4m3_to_f32

    acc = e4m3_to_f32(xq).astype(np.float64) @ e4m3_to_f32(np_bytes(q)).astype(np.float64).T
    want = ((acc.astype(np.float32) * xs[:, None]).astype(np.float32) * s.cpu().numpy()[None, :]).astype(np.float32)
    want = (want + np_values(b)[None, :]).astype(np.float32)
    close_bf16(y, want, f"fp8 {m}x{k}x{n}")
    golden_like = oq.fp8_w8a8_linear(np_values(x), np_bytes(q), s.cpu().numpy(), np_values(b), out_dtype="f32")
    close_bf16(y, golden_like, "fp8 vs dequant-matmul")


@pytest.mark.parametrize("m,k,n", [(44, 256, 128), (300, 1024, 512), (4096, 14336, 256), (130, 512, 3200)])
def test_mxfp8_linear(kq, m, k, n, golden):
    g = torch.Generator().manual_seed(m)
    x = torch.randn(m, k, generator=g).to(torch.bfloat16)
    w = (torch.randn(n, k, generator=g) * 0.015).to(torch.bfloat16)
    b = torch.randn(n, generator=g).to(torch.bfloat16)
    q, s = kq.quantize_mxfp8(w.to(DEV))
    y = kq.mxfp8_linear(x.to(DEV), q, s, b.to(DEV))
    rows = slice(0, min(m, 256))
    xq, xs = oq.quantize_mxfp8(np_values(x[rows]))
    acc = oq.mxfp8_linear_codes(xq, xs, np_bytes(q), np_bytes(s), None, out_dtype="f32")
    want = (bf16_to_f32(f32_to_bf16(acc)) + np_values(b)[None, :]).astype(np.float32)
    close_bf16(y[rows], want, f"mxfp8 {m}x{k}x{n}")
    gg = golden
    xl = torch.from_numpy(gg["mxl_x"].view(np.int16)).view(torch.bfloat16).to(DEV)
    wq = torch.from_numpy(gg["mxl_wq"]).view(torch.float8_e4m3fn).to(DEV)
    ws = torch.from_numpy(gg["mxl_ws"]).view(torch.float8_e8m0fnu).to(DEV)
    wb = torch.from_numpy(gg["mxl_bias"].view(np.int16)).view(torch.bfloat16).to(DEV)
    yl = kq.mxfp8_linear(xl, wq, ws, wb)
    # the golden output is the reference's CPU path (one rounding after the bias); the GPU
    # path it mirrors rounds the GEMM to bf16 before the bias: the comparator's tolerance
    close_bf16_tol(yl, bf16_to_f32(gg["mxl_y"]), "mxfp8 golden")


@pytest.mark.parametrize("m,k,n", [(48, 256, 128), (200, 1024, 384), (1024, 8192, 512), (130, 512, 3200),
                                   (256, 1024, 3264)])
def test_fp4_w4a4_linear(kq, m, k, n, golden):
    g = torch.Generator().manual_seed(n)
    x = torch.randn(m, k, generator=g).to(torch.bfloat16)
    w = (torch.randn(n, k, generator=g) * 0.01).to(torch.bfloat16)
    b = (torch.randn(n, generator=g) * 0.05).to(torch.bfloat16)
    q, s, ts = kq.quantize_fp4(w.to(DEV))
    y = kq.fp4_w4a4_linear(x.to(DEV), q, s, ts, b.to(DEV))
    rows = slice(0, min(m, 128))
    want = oq.fp4_w4a4_linear(np_values(x[rows]), np_bytes(q), np_bytes(s), float(ts), np_values(b), out_dtype="f32")
    close_bf16(y[rows], want, f"nvfp4 {m}x{k}x{n}")
    gg = golden
    xg = torch.from_numpy(gg["w4a4_x"].view(np.int16)).view(torch.bfloat16).to(DEV)
    qg = torch.from_numpy(gg["w4a4_q"]).to(DEV)
    sg = torch.from_numpy(gg["w4a4_s"]).view(torch.float8_e4m3fn).to(DEV)
    tg = torch.tensor(float(gg["w4a4_ts"]), device=DEV)
    bg = torch.from_numpy(gg["w4a4_bias"].view(np.int16)).view(torch.bfloat16).to(DEV)
    yg = kq.fp4_w4a4_linear(xg, qg, sg, tg, bg)
    ul = ulp_distance_bf16(np_bf16_bits(yg).reshape(-1), gg["w4a4_y"].reshape(-1))
    assert float(np.mean(ul <= 1)) >= 0.99 and ul.max() <= 4, (np.mean(ul == 0), ul.max())


@pytest.mark.parametrize("fmt,m,k,n", [("mxfp4", 64, 256, 128), ("mxfp4", 200, 1024, 384), ("mxfp4", 130, 96, 3200),
                                       ("mxfp4", 256, 2048, 3264), ("nvfp4", 70, 48, 256), ("nvfp4", 33, 4128, 192)])
def test_fp4_w4a4_linear_formats_and_ragged_k(kq, fmt, m, k, n):
    """MXFP4 (kind::mxf4nvf4 scale_vec::2X, e8m0 per 32) and K that is not a multiple of the
    GEMM's 256-element k-step (zero-padded codes and scales)."""
    g = torch.Generator().manual_seed(m * 7 + k)
    x = torch.randn(m, k, generator=g).to(torch.bfloat16)
    w = (torch.randn(n, k, generator=g) * 0.01).to(torch.bfloat16)
    b = (torch.randn(n, generator=g) * 0.05).to(torch.bfloat16)
    q, s, ts = kq.quantize_fp4(w.to(DEV), fmt)
    y = kq.fp4_w4a4_linear(x.to(DEV), q, s, ts, b.to(DEV), fmt=fmt)
    assert y.shape == (m, n) and y.dtype == torch.bfloat16
    rows = slice(0, min(m, 96))
    want = oq.fp4_w4a4_linear(np_values(x[rows]), np_bytes(q), np_bytes(s), float(ts), np_values(b), fmt=fmt,
                              out_dtype="f32")
    close_bf16(y[rows], want, f"{fmt} {m}x{k}x{n}")


def test_fp4_config4_row_sample(kq):
    """Config 4's shapes (K = 8192, N = 28672 sliced to 1024 output channels for the oracle)."""
    from kernel_agent_b200 import workloads

    x, w, b = workloads.config4(seed=0, device="cpu", n=1024)
    q, s, ts = kq.quantize_fp4(w.to(DEV))
    y = kq.fp4_w4a4_linear(x.to(DEV), q, s, ts, b.to(DEV))
    rows = [0, 1, 2, 8191]
    want = oq.fp4_w4a4_linear(np_values(x[rows]), np_bytes(q), np_bytes(s), float(ts), np_values(b), out_dtype="f32")
    close_bf16(y[rows], want, "config 4 rows")
    y2 = kq.fp4_w4a4_linear(x.to(DEV), q, s, ts, b.to(DEV))
    assert torch.equal(y, y2)  # deterministic


@pytest.fixture(scope="module")
def kb():
    from kernel_agent_b200.kernels import blockwise

    return blockwise


@pytest.mark.parametrize("m", [1, 16, 2048, 200, 5, 17, 32])
def test_fp8_blockwise_linear_config2(kb, m):
    """Config 2 (K = 1024, N = 3072, M in {1, 16, 2048}, plus a ragged M): against the oracle's
    per-128-K promotion of the same codes, and against the fp32 fake-quant matmul."""
    from kernel_agent_b200 import workloads
    from oracle import fp8lib

    x, w = workloads.config2(m, seed=m)
    bias = (torch.randn(3072, generator=torch.Generator().manual_seed(1)) * 0.1).to(torch.bfloat16)
    wq, ws = kb.quantize_fp8_blocks(w.to(DEV))
    for b in (None, bias):
        y = kb.fp8_blockwise_linear(x.to(DEV), wq, ws, None if b is None else b.to(DEV))
        assert y.shape == (m, 3072) and y.dtype == torch.bfloat16
        rows = slice(0, min(m, 64))
        xq, xs = fp8lib.quantize_fp8_groups(np_values(x[rows]), 128)
        want = fp8lib.fp8_blockwise_gemm(xq, xs, np_bytes(wq), ws.cpu().numpy(),
                                         None if b is None else np_values(b), out_dtype="f32")
        close_bf16(y[rows], want, f"blockwise m={m} bias={b is not None}")
    fq = fp8lib.e4m3_to_f32(xq).astype(np.float64) * np.repeat(xs, 128, axis=1)
    wfq = fp8lib.e4m3_to_f32(np_bytes(wq)).astype(np.float64) * np.repeat(np.repeat(ws.cpu().numpy(), 128, 0), 128, 1)
    dq = (fq @ wfq.T + np_values(bias)[None, :]).astype(np.float32)
    close_bf16_tol(y[rows], dq, "blockwise vs dequant-matmul")


@pytest.mark.parametrize("m,k,n", [(1, 128, 128), (3, 1152, 384), (16, 8192, 256), (32, 2048, 640),
                                   (24, 640, 128), (9, 9216, 256)])
@pytest.mark.parametrize("out", ["bf16", "f16", "f32"])
def test_fp8_blockwise_decode_sizes(kb, m, k, n, out):
    """The decode-size path (M <= 32: the K steps of each 128-channel panel split over a cluster
    of up to 8 CTAs, reduced in K order through distributed shared memory) at K from one step
    to 64 steps, a step count that does not divide by 8, and each output dtype, with bias,
    against the oracle's promotion of the same codes; K = 9216 (72 steps) takes the tiled
    kernel."""
    from oracle import fp8lib

    g = torch.Generator().manual_seed(m * 7 + k + n)
    x = torch.randn(m, k, generator=g).to(torch.bfloat16)
    w = (torch.randn(n, k, generator=g) * 0.02).to(torch.bfloat16)
    bias = (torch.randn(n, generator=g) * 0.1).to(torch.bfloat16)
    wq, ws = kb.quantize_fp8_blocks(w.to(DEV))
    dt = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}[out]
    y = kb.fp8_blockwise_linear(x.to(DEV), wq, ws, bias.to(DEV), out_dtype=dt)
    assert y.shape == (m, n) and y.dtype == dt
    xq, xs = fp8lib.quantize_fp8_groups(np_values(x), 128)
    want = fp8lib.fp8_blockwise_gemm(xq, xs, np_bytes(wq), ws.cpu().numpy(), np_values(bias), out_dtype="f32")
    if out == "bf16":
        close_bf16(y, want, f"blockwise decode m={m} k={k} n={n}")
    else:
        got = y.float().cpu().numpy().astype(np.float64)
        rel = np.linalg.norm(got - want) / np.linalg.norm(want)
        assert rel < (1e-3 if out == "f16" else 1e-5), (m, k, n, out, rel)


def test_fp8_blockwise_golden(kb, golden):
    """The reference research script's fake-quant tensors (fq_groups / fq_block): the GEMM of
    our codes equals their fp32 matmul within the bf16 tolerance."""
    g = golden
    xb = torch.from_numpy(g["bw_x"].view(np.int16)).view(torch.bfloat16).to(DEV)
    wb = torch.from_numpy(g["bw_w"].view(np.int16)).view(torch.bfloat16).to(DEV)
    wq, ws = kb.quantize_fp8_blocks(wb)
    y = kb.fp8_blockwise_linear(xb, wq, ws)
    want = (g["bw_x_fq"].astype(np.float64) @ g["bw_w_fq"].astype(np.float64).T).astype(np.float32)
    close_bf16_tol(y, want, "blockwise golden")
    y32 = kb.fp8_blockwise_linear(xb, wq, ws, out_dtype=torch.float32)
    rel = np.linalg.norm(y32.cpu().numpy() - want) / np.linalg.norm(want)
    assert rel < 1e-5, rel  # fp32 out: only the fp32 partial / promotion roundings differ


def test_fp8_blockwise_rejects_bad_shapes(kb):
    x = torch.randn(4, 200, device=DEV).to(torch.bfloat16)
    with pytest.raises(ValueError):
        kb.quantize_fp8_groups(x)
    from kernel_agent_b200.kernels import gemm

    a = torch.zeros(4, 256, dtype=torch.uint8, device=DEV).view(torch.float8_e4m3fn)
    b = torch.zeros(200, 256, dtype=torch.uint8, device=DEV).view(torch.float8_e4m3fn)
    with pytest.raises(ValueError, match="multiples of 128"):
        gemm.fp8_blockwise(a, torch.ones(4, 2, device=DEV), b, torch.ones(2, 2, device=DEV))


def test_gemm_status_clean():
    from kernel_agent_b200 import _native

    assert _native.device_status() == 0


# ------------------------------------------------------------------ decode sizes (M <= 32)
# kernel-agent's skinny W8A8 examples (agent/examples/cuda_int8_skinny_gemm.py,
# cuda_fp8_skinny_gemm.py): the weight streams through the tensor core, the tokens are the
# MMA's N. Same numerics as the tiled path: INT8 bit for bit, FP8 within the bf16 tolerance.

@pytest.mark.parametrize("m", [1, 3, 8, 16, 17, 31, 32])
@pytest.mark.parametrize("k,n", [(1024, 1024), (4096, 4160), (896, 200)])
def test_int8_w8a8_linear_decode_sizes(kq, m, k, n):
    g = torch.Generator().manual_seed(m * 131 + n)
    x = torch.randn(m, k, generator=g).to(torch.bfloat16)
    w = (torch.randn(n, k, generator=g) * 0.02).to(torch.bfloat16)
    b = (torch.randn(n, generator=g) * 0.1).to(torch.bfloat16)
    q, s = kq.quantize_int8(w.to(DEV))
    y = kq.int8_w8a8_linear(x.to(DEV), q, s, b.to(DEV))
    want = oq.int8_w8a8_linear(np_values(x), np_bytes(q).view(np.int8), s.cpu().numpy(), np_values(b))
    assert y.shape == (m, n) and np.array_equal(np_bf16_bits(y), want)
    a = rand_i8(g, m, k)
    got = kq.int8_matmul(a.to(DEV), q).cpu().numpy()
    assert np.array_equal(got, oq.int8_matmul(a.numpy(), np_bytes(q).view(np.int8)))


@pytest.mark.parametrize("m", [1, 16, 24, 32])
@pytest.mark.parametrize("k,n", [(1024, 3072), (4096, 4096)])
def test_fp8_w8a8_linear_decode_sizes(kq, m, k, n):
    g = torch.Generator().manual_seed(m + 3 * n)
    x = torch.randn(m, k, generator=g).to(torch.bfloat16)
    w = (torch.randn(n, k, generator=g) * 0.02).to(torch.bfloat16)
    b = (torch.randn(n, generator=g) * 0.1).to(torch.bfloat16)
    q, s = kq.quantize_fp8(w.to(DEV))
    y = kq.fp8_w8a8_linear(x.to(DEV), q, s, b.to(DEV))
    close_bf16(y, oq.fp8_w8a8_linear(np_values(x), np_bytes(q), s.cpu().numpy(), np_values(b), out_dtype="f32"),
               f"fp8 decode {m}x{k}x{n}")
