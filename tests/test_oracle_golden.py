"""The CPU oracle against the reference's golden vectors and known answers (no GPU).

The golden vectors are the reference's own outputs (``tests/golden/make_golden.py``); the
known answers are the ones the reference's tests pin (``tests/test_int8.py:47-48``,
``tests/test_mxfp8.py:29-36, 94``, ``tests/test_w4a4.py`` ties). Codes, scales and integer
results must be bit for bit; fp32 GEMM outputs, which the reference accumulates in its own
order, within one bf16 step.
"""

from __future__ import annotations

import re

import numpy as np
import pytest

from helpers import ulp_distance_bf16
from oracle import compare as ocmp
from oracle import fp8lib as ofp8
from oracle import quant as oq
from oracle.formats import (
    bf16_to_f32,
    e2m1_codes,
    e4m3_from_f32,
    e4m3_to_f32,
    f32_to_bf16,
)


def bf(g, key):
    return bf16_to_f32(g[key])


def bf16_close(a_bits, b_bits, max_ulps=1, frac=1.0):
    """bf16 bit patterns within ``max_ulps`` steps on at least ``frac`` of the elements."""
    a = a_bits.astype(np.int32)
    b = b_bits.astype(np.int32)
    # map sign-magnitude to a monotonic integer line
    a = np.where(a & 0x8000, -(a & 0x7FFF), a)
    b = np.where(b & 0x8000, -(b & 0x7FFF), b)
    d = np.abs(a - b)
    return float((d <= max_ulps).mean()) >= frac and int(d.max()) <= 4 * max_ulps


# ------------------------------------------------------------------ known answers


def test_known_answers_of_the_reference_tests():
    # INT8: codes round to nearest even (tests/test_int8.py:47-48)
    q, _ = oq.quantize_int8(np.array([[127.0, 2.5, 3.5, -2.5]], np.float32))
    assert q.tolist() == [[127, 2, 4, -2]]
    # MXFP8 exponent rules (tests/test_mxfp8.py:29-36)
    amax = np.array([0.0, 1e-40, 1.0, 224.0, 448.0, 449.0, 15.2, 3.0e38], np.float32)
    assert oq.mx_scale_exponents(amax, "ceil").tolist() == [-127, -127, -8, -1, 0, 1, -4, 120]
    assert oq.mx_scale_exponents(amax, "floor").tolist() == [-127, -127, -8, -1, 0, 0, -5, 119]
    # the swizzled offset (tests/test_mxfp8.py:94)
    assert oq.mx_scale_offset(33, 5, 8) == 512 + 1 * 16 + 1 * 4 + 1
    # e2m1 tie directions (tests/test_w4a4.py, quantiser refusals)
    ties = np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, -0.25, -5.0], np.float32)
    assert e2m1_codes(ties).tolist() == [0, 2, 2, 4, 4, 6, 6, 0, 14]
    # e4m3 round trip of every code (NaN aside) and the saturation boundary
    codes = np.array([c for c in range(256) if c & 0x7F != 0x7F], np.uint8)
    assert np.array_equal(e4m3_from_f32(e4m3_to_f32(codes)), codes)
    assert e4m3_from_f32(np.array([448.0, 464.0, 2.0**-10, 2.0**-10 * 3], np.float32)).tolist() == [
        0x7E, 0x7E, 0, 2]


def test_int8(golden):
    g = golden
    q, s = oq.quantize_int8_activations(bf(g, "int8_x"))
    assert np.array_equal(q, g["int8_xq"]) and np.array_equal(s, g["int8_xs"])
    q, s = oq.quantize_int8_activations(bf(g, "int8_x"), g["int8_smooth"])
    assert np.array_equal(q, g["int8_xq_smooth"]) and np.array_equal(s, g["int8_xs_smooth"])
    wq, ws = oq.quantize_int8(bf(g, "int8_w"))
    assert np.array_equal(wq, g["int8_wq"]) and np.array_equal(ws, g["int8_ws"])
    y = oq.int8_w8a8_linear(bf(g, "int8_x"), wq, ws, bf(g, "int8_bias"))
    assert np.array_equal(y, g["int8_y"])  # exact int32 products: bit for bit
    with pytest.raises(ValueError, match="non-finite"):
        oq.quantize_int8(np.full((2, 4), np.inf, np.float32))


def test_fp8_per_token_and_channel(golden):
    g = golden
    q, s = oq.quantize_fp8_activations(bf(g, "fp8_x"))
    assert np.array_equal(q, g["fp8_xq"]) and np.array_equal(s, g["fp8_xs"])
    wq, ws = oq.quantize_fp8(bf(g, "fp8_w"))
    assert np.array_equal(wq, g["fp8_wq"]) and np.array_equal(ws, g["fp8_ws"])
    y = oq.fp8_w8a8_linear(bf(g, "fp8_x")[1:], wq, ws, bf(g, "fp8_bias"))
    assert bf16_close(y, g["fp8_y"])


def test_mxfp8(golden):
    g = golden
    assert np.array_equal(oq.mx_scale_exponents(g["mx_amax"], "ceil"), g["mx_e_ceil"])
    assert np.array_equal(oq.mx_scale_exponents(g["mx_amax"], "floor"), g["mx_e_floor"])
    q, s = oq.quantize_mxfp8(bf(g, "mx_x"))
    assert np.array_equal(q, g["mx_q"]) and np.array_equal(s, g["mx_s"])
    q, s = oq.quantize_mxfp8(bf(g, "mx_x"), "floor")
    assert np.array_equal(q, g["mx_q_floor"]) and np.array_equal(s, g["mx_s_floor"])
    for rows, cols in ((352, 32), (22, 8), (200, 12), (128, 4)):
        flat = oq.swizzle_scales(g[f"swz_in_{rows}_{cols}"])
        assert np.array_equal(flat, g[f"swz_out_{rows}_{cols}"])
        assert np.array_equal(oq.unswizzle_scales(flat, rows, cols), g[f"swz_in_{rows}_{cols}"])
    wq, ws = oq.quantize_mxfp8(bf(g, "mxl_w"))
    assert np.array_equal(wq, g["mxl_wq"]) and np.array_equal(ws, g["mxl_ws"])
    y = oq.mxfp8_linear(bf(g, "mxl_x"), wq, ws, bf(g, "mxl_bias"))
    assert bf16_close(y, g["mxl_y"])


def test_silu_mul_then_mxfp8(golden):
    g = golden
    h = oq.silu_mul(bf(g, "silu_g"), bf(g, "silu_u"))
    hb = f32_to_bf16(h)
    # eager's exp and ours may differ by an fp32 ulp before the bf16 rounding
    assert float((hb == g["silu_h"]).mean()) >= 0.99 and bf16_close(hb, g["silu_h"])
    q, s = oq.quantize_mxfp8(bf(g, "silu_h"))
    assert np.array_equal(q, g["silu_hq"]) and np.array_equal(s, g["silu_hs"])


@pytest.mark.parametrize("gran", ["token", "tensor"])
def test_nvfp4_activations(golden, gran):
    g = golden
    q, s, o = oq.quantize_fp4_activations(bf(g, "fp4_x"), "nvfp4", gran)
    assert np.array_equal(q, g[f"nvfp4_{gran}_q"])
    assert np.array_equal(s, g[f"nvfp4_{gran}_s"])
    assert np.array_equal(o, g[f"nvfp4_{gran}_o"])


def test_mxfp4_and_fp4_weights(golden):
    g = golden
    q, s, o = oq.quantize_fp4_activations(bf(g, "mxfp4_x"), "mxfp4")
    assert np.array_equal(q, g["mxfp4_q"]) and np.array_equal(s, g["mxfp4_s"])
    assert (o == 1).all()
    for fmt in ("nvfp4", "mxfp4"):
        q, s, ts = oq.quantize_fp4(bf(g, "mxfp4_x"), fmt)
        assert np.array_equal(q, g[f"w{fmt}_q"]) and np.array_equal(s, g[f"w{fmt}_s"])
        assert np.float32(ts) == g[f"w{fmt}_ts"]


def test_w4a4_linear(golden):
    g = golden
    q, s, ts = oq.quantize_fp4(bf(g, "w4a4_w"))
    assert np.array_equal(q, g["w4a4_q"]) and np.array_equal(s, g["w4a4_s"])
    assert np.float32(ts) == g["w4a4_ts"]
    y = oq.fp4_w4a4_linear(bf(g, "w4a4_x"), q, s, ts, bf(g, "w4a4_bias"))
    assert bf16_close(y, g["w4a4_y"])


def test_blockwise_fp8(golden):
    g = golden
    xq, xs = ofp8.quantize_fp8_groups(bf(g, "bw_x"), 128)
    deq = (e4m3_to_f32(xq).reshape(24, 4, 128) * xs[..., None]).reshape(24, 512)
    assert np.array_equal(deq.astype(np.float32), g["bw_x_fq"])
    wq, ws = ofp8.quantize_fp8_blocks(bf(g, "bw_w"), 128)
    deq = (e4m3_to_f32(wq).reshape(2, 128, 4, 128) * ws[:, None, :, None]).reshape(256, 512)
    assert np.array_equal(deq.astype(np.float32), g["bw_w_fq"])


def test_fp8_attention(golden):
    g = golden
    y = ofp8.attention_fp8(bf(g, "att_q"), bf(g, "att_k"), bf(g, "att_v"), causal=True)
    assert bf16_close(f32_to_bf16(y), g["att_y"], max_ulps=1, frac=0.99)
    for key, causal in (("att2_y", True), ("att2_y_nc", False)):
        # the reference sums P V in fp32 (its own order), the oracle in float64: outputs near
        # zero may differ by many bf16 steps, so the bound is relative L2 plus the share of
        # elements within one step
        y = ofp8.attention_fp8(bf(g, "att2_q"), bf(g, "att2_k"), bf(g, "att2_v"), causal=causal)
        want = bf16_to_f32(g[key]).astype(np.float64)
        assert np.linalg.norm(y - want) / np.linalg.norm(want) < 5e-3, key
        steps = ulp_distance_bf16(f32_to_bf16(y).reshape(-1), g[key].reshape(-1))
        assert float((steps <= 1).mean()) >= 0.999, key
    ref = ofp8.sdpa_fp32(bf(g, "att2_q"), bf(g, "att2_k"), bf(g, "att2_v"), causal=True)
    assert np.allclose(ref, g["att2_y_fp32"], rtol=1e-4, atol=1e-5)


def _shape_of(error):
    """An error string with its numbers masked: the problems it names, not their digits."""
    return None if error is None else re.sub(r"[-+]?\d+(\.\d+)?(e[-+]?\d+)?", "#", error)


def test_comparator(golden, golden_meta):
    """Verdicts, the problems named, mismatch fractions and outlier ratios bit for bit; the
    figures reported from norms and dot products (cosine, relative L2, norm and element
    ratios), which torch sums in its own fp32 order, within that order's noise."""
    names = {"bfloat16": "bf16", "float16": "f16", "float32": "f32"}
    for case in golden_meta["compare"]:
        dt = case["dtype"]
        ref, new = golden[case["ref"]], golden[case["new"]]
        if dt in ("bfloat16",):
            ref, new = bf16_to_f32(ref), bf16_to_f32(new)
        rer = None
        if case["rer"] is not None:
            rer = golden[case["rer"]]
            rer = bf16_to_f32(rer) if dt == "bfloat16" else rer
        kind = names.get(dt, "int")
        kw = dict(case["kw"])
        kw.setdefault("tier", "exact")
        got = ocmp.compare_tensors(case["result"]["name"], ref, new, kind, rerounded=rer, **kw)
        want = case["result"]
        label = want["name"]
        assert got["ok"] == want["ok"], (label, got, want)
        assert _shape_of(got.get("error")) == _shape_of(want.get("error")), (label, got, want)
        for key in ("mismatch_frac", "max_err_ratio", "max_abs_err"):
            assert got.get(key) == want.get(key), (label, key, got, want)
        for key, tol in (("cosine", 2e-5), ("rel_l2", 2e-4), ("norm_ratio", 2e-5),
                         ("element_ratio", 2e-4), ("max_err_over_rms", 2e-4),
                         ("mean_abs_err", 1e-5), ("rounding_spread", 2e-5),
                         ("error_over_spread", 2e-3)):
            if key in want:
                assert abs(got[key] - want[key]) <= tol * max(1.0, abs(want[key])), (label, key, got[key], want[key])


def test_scale_checks(golden, golden_meta):
    for chk in golden_meta["checks"]:
        x = bf16_to_f32(golden[chk["input"]])
        if chk["kind"] == "mxfp8":
            _, s = oq.quantize_mxfp8(x, chk["rule"])
            got = oq.mxfp8_saturation(x, s)
        else:
            fmt = chk["fmt"]
            _, s, o = oq.quantize_fp4_activations(x, fmt)
            if chk.get("variant") == "trunc":
                s = golden["stress_fp4_trunc_scales"]
            got = oq.fp4_scale_check(x, s, o, fmt)
        assert got == chk["result"], (chk, got)


def test_rotation_and_bias_correction(golden):
    """hadamard_rotate (fp32 within a few units: torch's matmul orders its sums its own way),
    fp4_bias_correction, quantize_fp4(unbiased=True) and fp4_w4a4_linear with rotate / unbiased
    against the reference's CPU results."""
    g = golden
    x, w, b = bf(g, "rot_x"), bf(g, "rot_w"), bf(g, "rot_b")
    for block in (16, 128):
        got = oq.hadamard_rotate(x, block)
        want = g[f"rot_x{block}"]
        assert np.max(np.abs(got - want)) <= 1e-6 * np.max(np.abs(want)) * block
    for fmt in ("nvfp4", "mxfp4"):
        cx, sx, ox = oq.quantize_fp4_activations(x, fmt)
        c = oq.fp4_bias_correction(x, cx, sx, ox, fmt)
        assert np.array_equal(c, g[f"bc_{fmt}_x"]), fmt
        q, s, ts = oq.quantize_fp4(w, fmt, unbiased=True)
        assert np.array_equal(q, g[f"ub_{fmt}_q"]) and np.array_equal(s, g[f"ub_{fmt}_s"])
        assert np.array_equal(np.asarray(ts, np.float32).reshape(-1), g[f"ub_{fmt}_ts"].reshape(-1)), fmt
        y = oq.fp4_w4a4_linear(x, q, s, ts, b, fmt=fmt, unbiased=True)
        assert bf16_close(y, g[f"ub_{fmt}_y"], max_ulps=1, frac=0.99), fmt
        wrot = bf16_to_f32(f32_to_bf16(oq.hadamard_rotate(w, 16)))
        q, s, ts = oq.quantize_fp4(wrot, fmt)
        frac_q = float(np.mean(q == g[f"rot_{fmt}_wq"]))
        assert frac_q > 0.999, (fmt, frac_q)  # the rotation's last-unit differences can flip a code
        y = oq.fp4_w4a4_linear(x, g[f"rot_{fmt}_wq"], g[f"rot_{fmt}_ws"], g[f"rot_{fmt}_ts"], b, fmt=fmt, rotate=16)
        assert bf16_close(y, g[f"rot_{fmt}_y"], max_ulps=2, frac=0.98), fmt
