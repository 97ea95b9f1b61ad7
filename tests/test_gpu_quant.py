"""The quantise producers on the GPU against the oracle and the reference's golden vectors:
codes and scales bit for bit (INT8, FP8 per token / channel / 1 x 128 / 128 x 128, MXFP8,
NVFP4, MXFP4, swizzled layouts), the fused SiLU * up producers, ragged and edge-case
inputs, and the full-size configuration inputs on row samples."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from helpers import np_bf16_bits, np_bytes, np_values, to_bf16, ulp_distance_bf16
from oracle import fp8lib as ofp8
from oracle import quant as oq
from oracle.formats import bf16_to_f32, e4m3_to_f32

pytestmark = pytest.mark.gpu

DEV = "cuda"


@pytest.fixture(scope="module")
def kq():
    from kernel_agent_b200.kernels import quant

    return quant


@pytest.fixture(scope="module")
def kp():
    from kernel_agent_b200.kernels import producers

    return producers


def gen(seed, shape, spread=0.0):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(*shape, generator=g)
    if spread:
        x = x * torch.logspace(-spread, spread, shape[0])[:, None]
    return x.to(torch.bfloat16)


def edge_rows(k):
    """Rows that exercise the formats' corners: zero, tiny (bf16 subnormal), huge, ties."""
    x = gen(99, (8, k))
    x[0] = 0
    x[1] = x[1] * 1e-39
    x[2] = x[2] * 1e30
    x[3, : k // 2] = 0
    x[4, 0] = 300.0
    x[5] = torch.tensor([127.0, 2.5, 3.5, -2.5] * (k // 4))
    x[6] = x[6] * 2.0**-130
    return x


SHAPES = [(1, 64), (17, 256), (200, 1024), (129, 4096), (3, 16384), (2, 40960)]


@pytest.mark.parametrize("rows,k", SHAPES)
def test_int8_per_token_and_channel(kq, rows, k):
    x = torch.cat([gen(rows + k, (rows, k), spread=3), edge_rows(k)])
    q, s = kq.quantize_int8_activations(x.to(DEV))
    rq, rs = oq.quantize_int8_activations(np_values(x))
    assert np.array_equal(np_bytes(q).view(np.int8), rq) and np.array_equal(s.cpu().numpy(), rs)
    w = x[: max(rows, 8)]
    wq, ws = kq.quantize_int8(w.to(DEV))
    rwq, rws = oq.quantize_int8(np_values(w))
    assert np.array_equal(np_bytes(wq).view(np.int8), rwq) and np.array_equal(ws.cpu().numpy(), rws)


def test_int8_smooth_and_golden(kq, golden):
    g = golden
    x = torch.from_numpy(g["int8_x"].view(np.int16)).view(torch.bfloat16).to(DEV)
    q, s = kq.quantize_int8_activations(x)
    assert np.array_equal(np_bytes(q).view(np.int8), g["int8_xq"]) and np.array_equal(s.cpu().numpy(), g["int8_xs"])
    sm = torch.from_numpy(g["int8_smooth"]).to(DEV)
    q, s = kq.quantize_int8_activations(x, sm)
    assert np.array_equal(np_bytes(q).view(np.int8), g["int8_xq_smooth"])
    assert np.array_equal(s.cpu().numpy(), g["int8_xs_smooth"])
    w = torch.from_numpy(g["int8_w"].view(np.int16)).view(torch.bfloat16).to(DEV)
    wq, ws = kq.quantize_int8(w)
    assert np.array_equal(np_bytes(wq).view(np.int8), g["int8_wq"]) and np.array_equal(ws.cpu().numpy(), g["int8_ws"])
    rq, rs = oq.quantize_int8(np_values(w), np.linspace(0.5, 2, w.shape[1]).astype(np.float32))
    q, s = kq.quantize_int8(w, torch.from_numpy(np.linspace(0.5, 2, w.shape[1]).astype(np.float32)).to(DEV))
    assert np.array_equal(np_bytes(q).view(np.int8), rq) and np.array_equal(s.cpu().numpy(), rs)


@pytest.mark.parametrize("rows,k", SHAPES)
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_fp8_per_token(kq, rows, k, dtype):
    x = torch.cat([gen(rows * 3 + k, (rows, k), spread=4), edge_rows(k)]).to(dtype)
    if dtype == torch.float16:  # keep the huge row finite: inf / inf is a NaN whose sign
        x = torch.nan_to_num(x, posinf=6e4, neginf=-6e4)  # differs between devices
    q, s = kq.quantize_fp8_activations(x.to(DEV))
    rq, rs = oq.quantize_fp8_activations(np_values(x))
    assert np.array_equal(np_bytes(q), rq) and np.array_equal(s.cpu().numpy(), rs)


def test_fp8_golden(kq, golden):
    g = golden
    x = torch.from_numpy(g["fp8_x"].view(np.int16)).view(torch.bfloat16).to(DEV)
    q, s = kq.quantize_fp8_activations(x)
    assert np.array_equal(np_bytes(q), g["fp8_xq"]) and np.array_equal(s.cpu().numpy(), g["fp8_xs"])
    w = torch.from_numpy(g["fp8_w"].view(np.int16)).view(torch.bfloat16).to(DEV)
    q, s = kq.quantize_fp8(w)
    assert np.array_equal(np_bytes(q), g["fp8_wq"]) and np.array_equal(s.cpu().numpy(), g["fp8_ws"])
    with pytest.raises(ValueError, match="non-finite"):
        kq.quantize_fp8(torch.full((2, 8), float("inf"), device=DEV))


@pytest.mark.parametrize("rows,k,group", [(1, 1024, 128), (16, 1024, 128), (37, 512, 64), (5, 256, 32)])
def test_fp8_groups(rows, k, group):
    from kernel_agent_b200.kernels import blockwise

    x = torch.cat([gen(rows, (rows, k), spread=5), edge_rows(k)])
    q, s = blockwise.quantize_fp8_groups(x.to(DEV), group)
    rq, rs = ofp8.quantize_fp8_groups(np_values(x), group)
    assert np.array_equal(np_bytes(q), rq) and np.array_equal(s.cpu().numpy(), rs)


def test_fp8_blocks_and_golden(golden):
    from kernel_agent_b200.kernels import blockwise

    g = golden
    xb = torch.from_numpy(g["bw_x"].view(np.int16)).view(torch.bfloat16).to(DEV)
    q, s = blockwise.quantize_fp8_groups(xb, 128)
    deq = (e4m3_to_f32(np_bytes(q)).reshape(24, 4, 128) * s.cpu().numpy()[..., None]).reshape(24, 512)
    assert np.array_equal(deq.astype(np.float32), g["bw_x_fq"])
    wb = torch.from_numpy(g["bw_w"].view(np.int16)).view(torch.bfloat16).to(DEV)
    q, s = blockwise.quantize_fp8_blocks(wb, 128)
    deq = (e4m3_to_f32(np_bytes(q)).reshape(2, 128, 4, 128) * s.cpu().numpy()[:, None, :, None]).reshape(256, 512)
    assert np.array_equal(deq.astype(np.float32), g["bw_w_fq"])
    w = gen(5, (384, 1024)) * 0.02
    w[7, 300] = 40.0
    q, s = blockwise.quantize_fp8_blocks(w.to(DEV), 128)
    rq, rs = ofp8.quantize_fp8_blocks(np_values(w), 128)
    assert np.array_equal(np_bytes(q), rq) and np.array_equal(s.cpu().numpy(), rs)


def test_mx_exponents_golden(kq, golden):
    g = golden
    a = torch.from_numpy(g["mx_amax"]).to(DEV)
    assert np.array_equal(kq.mx_scale_exponents(a, "ceil").cpu().numpy(), g["mx_e_ceil"])
    assert np.array_equal(kq.mx_scale_exponents(a, "floor").cpu().numpy(), g["mx_e_floor"])


@pytest.mark.parametrize("rows,k", [(1, 32), (48, 256), (130, 4096), (7, 14336)])
@pytest.mark.parametrize("rule", ["ceil", "floor"])
def test_mxfp8(kq, rows, k, rule, golden):
    x = torch.cat([gen(rows + 7, (rows, k), spread=30), edge_rows(k)])
    q, s = kq.quantize_mxfp8(x.to(DEV), rule)
    rq, rs = oq.quantize_mxfp8(np_values(x), rule)
    assert np.array_equal(np_bytes(q), rq) and np.array_equal(np_bytes(s), rs)
    g = golden
    xm = torch.from_numpy(g["mx_x"].view(np.int16)).view(torch.bfloat16).to(DEV)
    q, s = kq.quantize_mxfp8(xm, rule)
    suffix = "" if rule == "ceil" else "_floor"
    assert np.array_equal(np_bytes(q), g["mx_q" + suffix]) and np.array_equal(np_bytes(s), g["mx_s" + suffix])


def test_swizzle_golden(kq, golden):
    for rows, cols in ((352, 32), (22, 8), (200, 12), (128, 4)):
        s = torch.from_numpy(golden[f"swz_in_{rows}_{cols}"]).to(DEV)
        flat = kq.swizzle_mx_scales(s.view(torch.float8_e8m0fnu))
        assert np.array_equal(np_bytes(flat), golden[f"swz_out_{rows}_{cols}"])


@pytest.mark.parametrize("rows,k", [(5, 256), (300, 1024), (64, 14336)])
def test_silu_mul_mxfp8_and_fp8(kp, kq, rows, k, golden):
    g = gen(rows, (rows, k)) * 3
    u = gen(rows + 1, (rows, k))
    h = torch.empty(rows, k, dtype=torch.bfloat16, device=DEV)
    q, s = kp.silu_mul_fp8(g.to(DEV), u.to(DEV), mx=True, out=h)
    # h: eager's math within one bf16 step of a correctly rounded exp (>= 99 % identical)
    ref_h = oq.silu_mul(np_values(g), np_values(u))
    from oracle.formats import f32_to_bf16

    d = ulp_distance_bf16(np_bf16_bits(h), f32_to_bf16(ref_h))
    assert float((d == 0).mean()) >= 0.99 and int(d.max()) <= 1
    # codes and scales: the quantisation of the kernel's own h, bit for bit
    rq, rs = oq.quantize_mxfp8(np_values(h))
    assert np.array_equal(np_bytes(q), rq) and np.array_equal(np_bytes(s), rs)
    # swizzled scales and the merged gate|up layout give the same bytes
    merged = torch.cat([g, u], dim=1).to(DEV)
    q2, s2 = kp.silu_mul_fp8(merged, mx=True, blocked=True)
    assert torch.equal(q2.view(torch.uint8), q.view(torch.uint8))
    assert np.array_equal(np_bytes(s2), oq.swizzle_scales(rs))
    # per-token FP8 of silu * up
    h2 = torch.empty_like(h)
    q3, s3 = kp.silu_mul_fp8(g.to(DEV), u.to(DEV), out=h2)
    assert torch.equal(h2, h)
    rq3, rs3 = oq.quantize_fp8_activations(np_values(h2))
    assert np.array_equal(np_bytes(q3), rq3) and np.array_equal(s3.cpu().numpy(), rs3)
    # the golden silu inputs: the reference's h within a step, codes of our h exact
    gg = golden
    gt = torch.from_numpy(gg["silu_g"].view(np.int16)).view(torch.bfloat16).to(DEV)
    ut = torch.from_numpy(gg["silu_u"].view(np.int16)).view(torch.bfloat16).to(DEV)
    hh = torch.empty_like(gt)
    kp.silu_mul_fp8(gt, ut, mx=True, out=hh)
    d = ulp_distance_bf16(np_bf16_bits(hh), gg["silu_h"])
    assert float((d == 0).mean()) >= 0.99 and int(d.max()) <= 1


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_silu_mul_matches_eager_on_gpu(kp, dtype):
    """The producer's SiLU(g) * u (a fast exponential checked against the rounding boundaries,
    the exact expf and IEEE division near them) against torch's own eager F.silu(g) * u on the
    GPU, x / (1 + expf(-x)) with an IEEE division: 4M elements over |g| <= 20 and the small
    values where the rounding boundaries are densest."""
    gen_ = torch.Generator(device=DEV).manual_seed(7)
    g = (torch.rand(1024, 4096, device=DEV, generator=gen_) * 40 - 20)
    g[:256] = torch.randn(256, 4096, device=DEV, generator=gen_) * 0.05
    g = g.to(dtype)
    u = torch.randn(1024, 4096, device=DEV, generator=gen_).to(dtype)
    h = torch.empty_like(g)
    kp.silu_mul_fp8(g, u, mx=True, out=h)
    eager = torch.nn.functional.silu(g) * u
    same = (h.view(torch.int16) == eager.view(torch.int16)).float().mean().item()
    assert same >= 0.9999, same
    assert torch.allclose(h.float(), eager.float(), rtol=2 ** -7, atol=0)


@pytest.mark.parametrize("gran", ["token", "tensor"])
def test_nvfp4_golden(kq, golden, gran):
    g = golden
    x = torch.from_numpy(g["fp4_x"].view(np.int16)).view(torch.bfloat16).to(DEV)
    q, s, o = kq.quantize_fp4_activations(x, "nvfp4", gran)
    assert np.array_equal(np_bytes(q), g[f"nvfp4_{gran}_q"])
    assert np.array_equal(np_bytes(s), g[f"nvfp4_{gran}_s"])
    assert np.array_equal(o.cpu().numpy(), g[f"nvfp4_{gran}_o"])


def test_mxfp4_and_fp4_weights_golden(kq, golden):
    g = golden
    x = torch.from_numpy(g["mxfp4_x"].view(np.int16)).view(torch.bfloat16).to(DEV)
    q, s, o = kq.quantize_fp4_activations(x, "mxfp4")
    assert np.array_equal(np_bytes(q), g["mxfp4_q"]) and np.array_equal(np_bytes(s), g["mxfp4_s"])
    for fmt in ("nvfp4", "mxfp4"):
        q, s, ts = kq.quantize_fp4(x, fmt)
        assert np.array_equal(np_bytes(q), g[f"w{fmt}_q"]) and np.array_equal(np_bytes(s), g[f"w{fmt}_s"])
        assert float(ts) == float(g[f"w{fmt}_ts"])


@pytest.mark.parametrize("rows,k", [(1, 16), (33, 64), (257, 1024), (64, 8192), (5, 6144), (3, 32768)])
@pytest.mark.parametrize("fmt", ["nvfp4", "mxfp4"])
def test_fp4_random(kq, rows, k, fmt):
    if k % kq.FP4_FORMATS[fmt][0]:
        pytest.skip("K is not a whole number of this format's blocks")
    x = torch.cat([gen(rows * 5 + k, (rows, k), spread=20), edge_rows(k)])
    for gran in (("token", "tensor") if fmt == "nvfp4" else ("token",)):
        q, s, o = kq.quantize_fp4_activations(x.to(DEV), fmt, gran)
        rq, rs, ro = oq.quantize_fp4_activations(np_values(x), fmt, gran)
        assert np.array_equal(np_bytes(q), rq) and np.array_equal(np_bytes(s), rs)
        assert np.array_equal(o.cpu().numpy(), ro)
    w = x[: max(8, rows)].clone()
    w[1] = 0
    q, s, ts = kq.quantize_fp4(w.to(DEV), fmt)
    rq, rs, rts = oq.quantize_fp4(np_values(w), fmt)
    assert np.array_equal(np_bytes(q), rq) and np.array_equal(np_bytes(s), rs) and float(ts) == float(rts)


def test_fp4_values_and_swizzle(kq):
    x = gen(3, (200, 512), spread=2)
    q, s, o = kq.quantize_fp4_activations(x.to(DEV))
    v = kq.fp4_values(q, s)
    assert np.array_equal(v.cpu().numpy(), oq.fp4_values(np_bytes(q), np_bytes(s)))
    flat = kq.swizzle_fp4_scales(s)
    assert flat.dtype == torch.float8_e4m3fn
    assert np.array_equal(np_bytes(flat), oq.swizzle_scales(np_bytes(s)))


@pytest.mark.parametrize("rows,k", [(4, 256), (130, 3072)])
def test_silu_mul_fp4(kp, rows, k):
    g = gen(rows + 11, (rows, k)) * 2
    u = gen(rows + 12, (rows, k))
    h = torch.empty(rows, k, dtype=torch.bfloat16, device=DEV)
    q, s, o = kp.silu_mul_fp4(g.to(DEV), u.to(DEV), out=h)
    rq, rs, ro = oq.quantize_fp4_activations(np_values(h))
    assert np.array_equal(np_bytes(q), rq) and np.array_equal(np_bytes(s), rs)
    assert np.array_equal(o.cpu().numpy(), ro)
    q2, s2, o2 = kp.silu_mul_fp4(g.to(DEV), u.to(DEV), swizzle=True)
    assert torch.equal(q2, q) and np.array_equal(np_bytes(s2), oq.swizzle_scales(rs))


def test_config_inputs_row_samples(kq, kp):
    """The full-size producer inputs of configs 3 and 4, quantised whole on the GPU, checked on
    row samples against the oracle; the codes' checksum does not change between calls."""
    from kernel_agent_b200 import workloads

    x, _, _ = workloads.config4(seed=0, device="cpu", n=128)
    q, s, o = kq.quantize_fp4_activations(x.to(DEV))
    rows = [0, 1, 4095, 8191]
    rq, rs, ro = oq.quantize_fp4_activations(np_values(x[rows]))
    assert np.array_equal(np_bytes(q[rows]), rq) and np.array_equal(np_bytes(s[rows]), rs)
    q2, s2, _ = kq.quantize_fp4_activations(x.to(DEV))
    assert torch.equal(q, q2) and torch.equal(s.view(torch.uint8), s2.view(torch.uint8))
    g, u, _ = workloads.config3(seed=0, device="cpu", h=128)
    h = torch.empty_like(g, device=DEV)
    q, s = kp.silu_mul_fp8(g.to(DEV), u.to(DEV), mx=True, out=h)
    rows = [0, 17, 4095]
    rq, rs = oq.quantize_mxfp8(np_values(h[rows]))
    assert np.array_equal(np_bytes(q[rows]), rq) and np.array_equal(np_bytes(s[rows]), rs)


def test_cpu_tensors_are_refused(kq):
    with pytest.raises(ValueError, match="CUDA tensor required"):
        kq.quantize_fp8_activations(torch.zeros(2, 16))
    with pytest.raises(ValueError, match="multiple of the MXFP8 block"):
        kq.quantize_mxfp8(torch.zeros(2, 48, device=DEV))
    with pytest.raises(ValueError, match="unknown FP4 format"):
        kq.quantize_fp4_activations(torch.zeros(2, 32, device=DEV), "int4")
    with pytest.raises(ValueError, match="granularity"):
        kq.quantize_fp4_activations(torch.zeros(2, 32, device=DEV), granularity="channel")
    e = kq.quantize_fp4_activations(torch.zeros(0, 32, device=DEV))
    assert [tuple(t.shape) for t in e] == [(0, 16), (0, 2), (0,)]


def _near(values: np.ndarray, ulps: int = 6) -> np.ndarray:
    """fp32 values within +-ulps units in the last place of each of ``values``."""
    v = values.astype(np.float32)
    out = [v]
    up, down = v.copy(), v.copy()
    for _ in range(ulps):
        up = np.nextafter(up, np.float32(np.inf))
        down = np.nextafter(down, np.float32(-np.inf))
        out += [up, down]
    return np.concatenate(out)


def _rows_of(values: np.ndarray, lead: float, width: int) -> np.ndarray:
    """Rows of ``width`` fp32 elements: ``lead`` first (the row's amax), then ``values``
    (padded with zeros)."""
    per = width - 1
    n = -(-values.size // per)
    body = np.zeros(n * per, np.float32)
    body[: values.size] = values
    rows = np.concatenate([np.full((n, 1), lead, np.float32), body.reshape(n, per)], axis=1)
    return rows


def test_rounding_boundaries_fp8_int8(kq):
    """Quotients within a few ulps of every rounding boundary (e4m3 midpoints, k + 1/2):
    the fast reciprocal path with its exact fallback gives the IEEE-division codes."""
    from oracle.formats import e4m3_to_f32

    e4 = np.sort(e4m3_to_f32(np.arange(0, 127, dtype=np.uint8)).astype(np.float64))
    mids = (e4[:-1] + e4[1:]) / 2
    for lead in (448.0 * 1.3, 448.0 * 0.77, 3.1e-3, 1.7e5):
        sc = np.float32(np.float32(lead) / np.float32(448.0))
        vals = _near(np.concatenate([mids, -mids]) * np.float64(sc))
        x = torch.from_numpy(_rows_of(vals, lead, 1024))
        q, s = kq.quantize_fp8_activations(x.to(DEV))
        rq, rs = oq.quantize_fp8_activations(x.numpy())
        assert np.array_equal(np_bytes(q), rq) and np.array_equal(s.cpu().numpy(), rs), lead
    halves = np.arange(0, 127) + 0.5
    for lead in (127.0 * 1.3, 0.91, 2.2e4):
        sc = np.float32(np.float32(lead) * oq.INT8_STEP)
        vals = _near(np.concatenate([halves, -halves]) * np.float64(sc))
        x = torch.from_numpy(_rows_of(vals, lead, 1024))
        q, s = kq.quantize_int8_activations(x.to(DEV))
        rq, rs = oq.quantize_int8_activations(x.numpy())
        assert np.array_equal(np_bytes(q).view(np.int8), rq) and np.array_equal(s.cpu().numpy(), rs), lead


@pytest.mark.parametrize("fmt", ["nvfp4", "mxfp4"])
def test_rounding_boundaries_fp4(kq, fmt):
    """e2m1 midpoints (0.25 ... 5) times each block's step, +-6 ulps: codes equal the
    oracle's (IEEE division), activations and weights."""
    block = kq.FP4_FORMATS[fmt][0]
    mids = np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0])
    g = np.random.default_rng(7)
    k = 64 * block
    lead = np.float32(13.37)
    maxima = (lead * g.uniform(0.02, 1.0, size=k // block)).astype(np.float32)
    maxima[0] = lead
    skel = np.zeros((1, k), np.float32)
    skel[0, ::block] = maxima
    _, rs, ro = oq.quantize_fp4_activations(skel, fmt, "token")
    from oracle.formats import e4m3_to_f32

    if fmt == "nvfp4":
        steps = (e4m3_to_f32(rs.reshape(-1)) * ro[0]).astype(np.float32)
    else:
        steps = np.ldexp(np.float32(1.0), rs.reshape(-1).astype(np.int32) - 127).astype(np.float32)
    row = skel.copy()
    for b in range(k // block):
        pool = _near(np.concatenate([mids, -mids]) * np.float64(steps[b]), ulps=2)
        cand = np.roll(pool, -b * (block - 1))[: block - 1]
        row[0, b * block + 1 : (b + 1) * block] = cand
    x = torch.from_numpy(np.repeat(row, 3, axis=0))
    q, s, o = kq.quantize_fp4_activations(x.to(DEV), fmt, "token")
    rq, rs2, ro2 = oq.quantize_fp4_activations(x.numpy(), fmt, "token")
    assert np.array_equal(np_bytes(q), rq) and np.array_equal(np_bytes(s), rs2)
    q, s, ts = kq.quantize_fp4(x.to(DEV), fmt)
    rq, rs2, rts = oq.quantize_fp4(x.numpy(), fmt)
    assert np.array_equal(np_bytes(q), rq) and np.array_equal(np_bytes(s), rs2)
