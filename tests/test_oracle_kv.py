"""The FP8 KV-cache oracle against the reference's golden vectors (no GPU), and the package's
host-side logic for the KV cache (``kv_cache_share``, argument checks that need no device).

The golden vectors are the reference's own outputs (``tests/golden/make_golden_kv.py``,
``kernel_agent.kernels.kv_quant``). Codes and scales must match bit for bit; the attention,
which the reference computes in fp32 in its own order, within 2e-6 relative L2.
"""

from __future__ import annotations

import json

import numpy as np
import pytest
import torch

from conftest import GOLDEN
from oracle import kv_quant as okv
from oracle.formats import bf16_to_f32, e4m3_to_f32


@pytest.fixture(scope="module")
def kvg():
    with np.load(GOLDEN / "kv_golden.npz") as z:
        return {k: z[k] for k in z.files}


@pytest.fixture(scope="module")
def kvmeta():
    return json.loads((GOLDEN / "kv_golden.json").read_text())


def f16_values(bits: np.ndarray) -> np.ndarray:
    return bits.view(np.float16).astype(np.float32)


@pytest.mark.parametrize("case,decode", [("q_bf16", bf16_to_f32), ("q_f32", None), ("q_f16", f16_values)])
def test_quantize_fp8_kv_bit_exact(kvg, case, decode):
    x = kvg[f"{case}_x"]
    x = decode(x) if decode else x
    codes, scales = okv.quantize_fp8_kv(x)
    assert np.array_equal(scales.view(np.uint32), kvg[f"{case}_scales"].view(np.uint32))
    assert np.array_equal(codes, kvg[f"{case}_codes"])


def test_quantize_fp8_kv_edge_rows(kvg):
    """The rows the golden case plants: zero (scale 1, codes 0), NaN (scale 1), inf (scale inf),
    and an f32 row whose amax / 448 underflows (the reference keeps the zero scale)."""
    x = bf16_to_f32(kvg["q_bf16_x"])
    codes, scales = okv.quantize_fp8_kv(x)
    assert scales[0, 1, 5] == 1.0 and not codes[0, 1, 5].any()
    assert scales[1, 0, 2] == 1.0 and (codes[1, 0, 2, 3] & 0x7F) == 0x7F
    assert np.isinf(scales[1, 1, 4])
    x32 = kvg["q_f32_x"]
    _, s32 = okv.quantize_fp8_kv(x32)
    assert s32[0, 1] == 0.0 and s32[2, 2] == 1.0


def test_dequantize_round_trip(kvg):
    codes, scales = kvg["q_bf16_codes"], kvg["q_bf16_scales"]
    deq = okv.dequantize_fp8_kv(codes, scales)
    with np.errstate(invalid="ignore", over="ignore"):
        want = e4m3_to_f32(codes) * scales[..., None]
    assert np.array_equal(np.nan_to_num(deq), np.nan_to_num(want.astype(np.float32)))


def rel(a, b) -> float:
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / np.linalg.norm(b))


def test_attention_against_the_reference(kvg):
    g = kvg
    out = okv.fp8_kv_attention(g["att_q"], g["att_kc"], g["att_ks"], g["att_vc"], g["att_vs"])
    assert rel(out, g["att_out"]) < 2e-6
    masked = okv.fp8_kv_attention(g["att_q"], g["att_kc"], g["att_ks"], g["att_vc"], g["att_vs"], scale=0.1,
                                  lengths=g["att_lengths"])
    assert rel(masked, g["att_masked"]) < 2e-6
    # a sequence of one valid token: its output is that token's V
    v1 = okv.dequantize_fp8_kv(g["att_vc"][1, :, :1], g["att_vs"][1, :, :1])
    assert np.allclose(masked[1, :4, 0], v1[0, 0], atol=1e-6) and np.allclose(masked[1, 4:, 0], v1[1, 0], atol=1e-6)


def test_attention_several_queries_bf16(kvg):
    g = kvg
    out = okv.fp8_kv_attention(bf16_to_f32(g["att2_q"]), g["att2_kc"], g["att2_ks"], g["att2_vc"], g["att2_vs"])
    want = bf16_to_f32(g["att2_out"])
    assert rel(bf16_to_f32(np.asarray(torch.from_numpy(out).to(torch.bfloat16).view(torch.int16).numpy()
                                      .view(np.uint16))), want) < 4e-3


def test_error_report(kvg, kvmeta):
    k = bf16_to_f32(kvg["err_k"])
    rep = okv.fp8_kv_error(k, k * np.float32(0.5))
    want = kvmeta["error"]
    for key in ("k_rel_l2", "k_worst_row_rel_l2", "v_rel_l2", "v_worst_row_rel_l2"):
        assert rep[key] == pytest.approx(want[key], abs=2e-5), key
    assert okv.fp8_kv_bytes(k.shape, 2) == want["bytes"]


def test_kv_cache_share(kvmeta):
    got = okv.kv_cache_share(batch=8, tokens=8192, layers=28, kv_heads=8, head_dim=128, other_bytes=16e9)
    assert got == pytest.approx(kvmeta["share"], rel=1e-12)
    small = okv.kv_cache_share(batch=1, tokens=77, layers=2, kv_heads=2, head_dim=64, other_bytes=0.0,
                               elem_bytes=4.0)
    assert small == pytest.approx(kvmeta["share_small"], rel=1e-12)


def test_package_share_and_cpu_refusal(kvmeta):
    from kernel_agent_b200.kernels import kv_quant as kv

    got = kv.kv_cache_share(batch=8, tokens=8192, layers=28, kv_heads=8, head_dim=128, other_bytes=16e9)
    assert got == pytest.approx(kvmeta["share"], rel=1e-12)
    with pytest.raises(ValueError, match="CUDA"):
        kv.quantize_fp8_kv(torch.zeros(2, 64))
    with pytest.raises(ValueError, match="head_dim"):
        kv.quantize_fp8_kv(torch.zeros(2, 48))
    with pytest.raises(ValueError, match="CUDA"):
        kv.Fp8KVCache(1, 1, 8, 64, device="cpu")
