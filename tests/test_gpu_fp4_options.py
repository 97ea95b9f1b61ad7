"""The W4A4 options on the GPU: the block Hadamard rotation, the per-row bias correction,
``quantize_fp4(unbiased=True)`` and ``fp4_w4a4_linear`` with ``rotate`` / ``unbiased``, against
the reference's CPU results (golden)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from helpers import np_bf16_bits, np_bytes, ulp_distance_bf16
from oracle.formats import bf16_to_f32

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(scope="module")
def kq():
    from kernel_agent_b200.kernels import quant

    return quant


def bf(g, key):
    return torch.from_numpy(g[key].view(np.int16)).view(torch.bfloat16).to(DEV)


def f32_ulps(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    ia, ib = a.astype(np.float32).view(np.int32).astype(np.int64), b.astype(np.float32).view(np.int32).astype(np.int64)
    return np.abs(ia - ib)


def test_hadamard_rotate(kq, golden):
    x = bf(golden, "rot_x")
    for block in (16, 128):
        got = kq.hadamard_rotate(x, block).cpu().numpy()
        want = golden[f"rot_x{block}"]
        assert np.max(np.abs(got - want)) <= 1e-6 * np.max(np.abs(want)) * block, block
    h = kq.hadamard(8)
    assert torch.allclose(h @ h, torch.eye(8), atol=1e-6)
    with pytest.raises(ValueError, match="power of two"):
        kq.hadamard_rotate(x[:, :48], 24)
    with pytest.raises(ValueError, match="not a multiple of the rotation"):
        kq.hadamard_rotate(x, 24)


@pytest.mark.parametrize("fmt", ["nvfp4", "mxfp4"])
def test_bias_correction_and_unbiased(kq, golden, fmt):
    g = golden
    x, w, b = bf(g, "rot_x"), bf(g, "rot_w"), bf(g, "rot_b")
    cx, sx, ox = kq.quantize_fp4_activations(x, fmt)
    c = kq.fp4_bias_correction(x, cx, sx, ox).cpu().numpy()
    assert f32_ulps(c, g[f"bc_{fmt}_x"]).max() <= 1, fmt  # float64 sums in another order
    q, s, ts = kq.quantize_fp4(w, fmt, unbiased=True)
    assert np.array_equal(np_bytes(q), g[f"ub_{fmt}_q"]) and np.array_equal(np_bytes(s), g[f"ub_{fmt}_s"])
    assert f32_ulps(ts.cpu().numpy().reshape(-1), g[f"ub_{fmt}_ts"].reshape(-1)).max() <= 1
    y = kq.fp4_w4a4_linear(x, q, s, ts, b, fmt=fmt, unbiased=True)
    d = ulp_distance_bf16(np_bf16_bits(y).reshape(-1), g[f"ub_{fmt}_y"].reshape(-1))
    assert float(np.mean(d <= 1)) >= 0.99 and int(d.max()) <= 4, (fmt, float(np.mean(d == 0)), int(d.max()))


@pytest.mark.parametrize("fmt", ["nvfp4", "mxfp4"])
def test_rotated_linear(kq, golden, fmt):
    g = golden
    x, b = bf(g, "rot_x"), bf(g, "rot_b")
    q = torch.from_numpy(g[f"rot_{fmt}_wq"]).to(DEV)
    dt = torch.float8_e4m3fn if fmt == "nvfp4" else torch.float8_e8m0fnu
    s = torch.from_numpy(g[f"rot_{fmt}_ws"]).view(dt).to(DEV)
    ts = torch.tensor(float(g[f"rot_{fmt}_ts"]), device=DEV)
    y = kq.fp4_w4a4_linear(x, q, s, ts, b, fmt=fmt, rotate=16)
    got = np.asarray(y.float().cpu().numpy(), np.float64)
    want = bf16_to_f32(g[f"rot_{fmt}_y"]).astype(np.float64)
    rel = np.linalg.norm(got - want) / np.linalg.norm(want)
    d = ulp_distance_bf16(np_bf16_bits(y).reshape(-1), g[f"rot_{fmt}_y"].reshape(-1))
    # the rotation's last-unit differences can flip an activation code: tolerance-level parity
    assert rel < 5e-3 and float(np.mean(d <= 1)) >= 0.98, (fmt, rel, float(np.mean(d <= 1)))
