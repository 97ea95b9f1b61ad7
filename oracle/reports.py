"""CPU restatement of the reference's numerical error reports (test infrastructure only).

Reference: ``src/kernel_agent/kernels/quant.py`` (kernel-agent 0.1.0): ``_error_metrics``
302-326, ``fp8_error`` 133-181, ``fp4_error`` 328-359, ``fp8_w8a8_error`` 420-476,
``mxfp8_error`` 707-768, ``int8_error`` 926-949, ``int8_w8a8_error`` 951-1000,
``smoothquant_factors`` 1002-1041, ``fp4_saturation`` 1260-1297 and ``fp4_w4a4_error``
1511-1573. Sums and products are float64 (the reference reduces in fp32 in torch's order);
the reports round to the reference's digits, so they match its values to about the last
printed digit (pinned by ``tests/golden/reports_golden.json``).
"""

from __future__ import annotations

import math

import numpy as np

from . import quant as oq
from .formats import F32, e4m3_to_f32, f32

_ERR = {"over": "ignore", "invalid": "ignore", "divide": "ignore", "under": "ignore"}


def _sig(value: float, digits: int = 4) -> float:
    """quant.py:129-130."""
    return float(f"{value:.{digits}g}") if math.isfinite(value) else value


def _weight_fields(w: np.ndarray, deq: np.ndarray) -> dict:
    """quant.py:305-318: rel_l2, worst_channel_rel_l2, underflow, crest."""
    w, deq = w.astype(np.float64), deq.astype(np.float64)
    diff = w - deq
    norm = float(np.sqrt((w * w).sum()))
    row_norm = np.sqrt((w * w).sum(axis=1))
    row_err = np.sqrt((diff * diff).sum(axis=1)) / np.maximum(row_norm, 1e-30)
    nonzero = w != 0
    rms = row_norm / math.sqrt(max(w.shape[1], 1))
    crest = np.abs(w).max(axis=1) / np.maximum(rms, 1e-30)
    live = row_norm > 0
    return {
        "rel_l2": _sig(float(np.sqrt((diff * diff).sum())) / norm if norm > 0 else 0.0),
        "worst_channel_rel_l2": _sig(float(row_err[live].max()) if norm > 0 else 0.0),
        "underflow": _sig(float((nonzero & (deq == 0)).sum()) / max(int(nonzero.sum()), 1)),
        "crest": _sig(float(crest[live].max()) if norm > 0 else 0.0),
    }


def _output_fields(ref: np.ndarray, new: np.ndarray) -> dict:
    """quant.py:320-325, 460-472, 1552-1571: the output error of ``new`` against ``ref``."""
    ref, new = ref.astype(np.float64), new.astype(np.float64)
    ref_norm, new_norm = float(np.linalg.norm(ref)), float(np.linalg.norm(new))
    dot = float((ref * new).sum())
    cos = dot / (ref_norm * new_norm) if ref_norm and new_norm else 1.0
    return {
        "output_rel_l2": _sig(float(np.linalg.norm(ref - new)) / ref_norm if ref_norm else 0.0),
        "output_cosine": round(cos, 6),
        "output_norm_ratio": round(new_norm / ref_norm, 5) if ref_norm else 1.0,
        "output_gain": round(dot / ref_norm**2, 5) if ref_norm else 1.0,
    }


def _activation_fields(a: np.ndarray, a_hat: np.ndarray) -> dict:
    """quant.py:455-469: activation_rel_l2, activation_crest, activation_underflow."""
    a, a_hat = a.astype(np.float64), a_hat.astype(np.float64)
    norm = float(np.linalg.norm(a))
    rms = np.sqrt((a * a).mean(axis=1))
    crest = np.abs(a).max(axis=1) / np.maximum(rms, 1e-30)
    nonzero = a != 0
    return {
        "activation_rel_l2": _sig(float(np.linalg.norm(a - a_hat)) / norm if norm > 0 else 0.0),
        "activation_crest": _sig(float(crest[rms > 0].max()) if (rms > 0).any() else 0.0),
        "activation_underflow": _sig(float((nonzero & (a_hat == 0)).sum()) / max(int(nonzero.sum()), 1)),
    }


def _with_output(report: dict, w, deq, x) -> dict:
    if x is not None:
        a = f32(x).reshape(-1, w.shape[1]).astype(np.float64)
        out = _output_fields(a @ w.astype(np.float64).T, a @ deq.astype(np.float64).T)
        report["output_rel_l2"] = out["output_rel_l2"]
        report["output_cosine"] = out["output_cosine"]
    return report


def fp8_error(weight, element_bytes: int, x=None) -> dict:
    """quant.py:133-181 (e4m3 per output channel)."""
    w = f32(weight)
    q, s = oq.quantize_fp8(w)
    deq = (e4m3_to_f32(q) * s[:, None]).astype(F32)
    rep = {"format": "float8_e4m3fn", "granularity": "per output channel", **_weight_fields(w, deq),
           "bytes": {"before": w.size * element_bytes, "after": q.size + 4 * s.size}}
    return _with_output(rep, w, deq, x)


def int8_error(weight, element_bytes: int, x=None, smooth=None) -> dict:
    """quant.py:926-949."""
    w = f32(weight)
    q, s = oq.quantize_int8(w, smooth)
    if smooth is not None:
        w = (w * f32(smooth)[None, :]).astype(F32)
    deq = (q.astype(F32) * s[:, None]).astype(F32)
    rep = {"format": "int8", "granularity": "per output channel, symmetric (amax / 127)",
           **_weight_fields(w, deq), "bytes": {"before": w.size * element_bytes, "after": q.size + 4 * s.size}}
    return _with_output(rep, w, deq, x)


def fp4_error(weight, element_bytes: int, fmt="nvfp4", x=None, unbiased=False) -> dict:
    """quant.py:328-359."""
    w = f32(weight)
    codes, scales, ts = oq.quantize_fp4(w, fmt, unbiased)
    ts = np.asarray(ts, np.float32)
    v = oq.fp4_values(codes, scales, fmt)
    deq = (v * (ts.reshape(-1, 1) if ts.size > 1 else ts.reshape(()))).astype(F32)
    block = oq.FP4_BLOCKS[fmt]
    kind = "e4m3 scale per {} + fp32 tensor scale" if fmt == "nvfp4" else "e8m0 scale per {}"
    nts = ts.size
    if nts > 1:
        kind += " x fp32 per channel (unbiased)"
    rep = {"format": fmt, "granularity": kind.format(block), **_weight_fields(w, deq),
           "bytes": {"before": w.size * element_bytes, "after": codes.size + scales.size + 4 * nts}}
    return _with_output(rep, w, deq, x), (codes, scales, ts)


def fp8_w8a8_error(weight, element_bytes: int, x) -> dict:
    """quant.py:420-476."""
    w = f32(weight)
    rep = fp8_error(w, element_bytes)
    q, s = oq.quantize_fp8(w)
    a = f32(x).reshape(-1, w.shape[1])
    xq, xs = oq.quantize_fp8_activations(a)
    a_hat = (e4m3_to_f32(xq) * xs[:, None]).astype(F32)
    deq = (e4m3_to_f32(q) * s[:, None]).astype(F32)
    out = _output_fields(a.astype(np.float64) @ w.astype(np.float64).T,
                         a_hat.astype(np.float64) @ deq.astype(np.float64).T)
    rep.update(activations="e4m3 per token", **_activation_fields(a, a_hat),
               output_rel_l2=out["output_rel_l2"], output_cosine=out["output_cosine"],
               output_norm_ratio=out["output_norm_ratio"])
    return rep


def int8_w8a8_error(weight, element_bytes: int, x, smooth=None) -> dict:
    """quant.py:951-1000."""
    w = f32(weight)
    a = f32(x).reshape(-1, w.shape[1])
    rep = int8_error(w, 4, smooth=smooth)  # quant.py:980: the report of the fp32 weight
    q, s = oq.quantize_int8(w, smooth)
    xq, xs = oq.quantize_int8_activations(a, smooth)
    a_hat = (xq.astype(F32) * xs[:, None]).astype(F32)
    if smooth is not None:
        a_hat = (a_hat * f32(smooth)[None, :]).astype(F32)
    acc = xq.astype(np.float64) @ q.astype(np.float64).T
    new = (acc * xs.astype(np.float64)[:, None] * s.astype(np.float64)[None, :]).astype(F32)
    out = _output_fields(a.astype(np.float64) @ w.astype(np.float64).T, new)
    rep.update(activations="int8 per token" + (" (SmoothQuant)" if smooth is not None else ""),
               **_activation_fields(a, a_hat), output_rel_l2=out["output_rel_l2"],
               output_cosine=out["output_cosine"], output_norm_ratio=out["output_norm_ratio"])
    return rep


def smoothquant_factors(act_amax, weight, alpha: float = 0.5) -> np.ndarray:
    """quant.py:1002-1041 (fp32 pow in float64, rounded once)."""
    a = f32(act_amax).reshape(-1)
    w = np.abs(f32(weight)).max(axis=0)
    ok = (a > 0) & (w > 0) & np.isfinite(a)
    with np.errstate(**_ERR):
        s = (np.maximum(a, 1e-30).astype(np.float64) ** alpha
             / np.maximum(w, 1e-30).astype(np.float64) ** (1.0 - alpha)).astype(F32)
    return np.where(ok, np.clip(s, 1e-5, 1e5), F32(1.0)).astype(F32)


def mxfp8_error(weight, element_bytes: int, x=None, rule="ceil") -> dict:
    """quant.py:707-768."""
    w = f32(weight)
    q, s = oq.quantize_mxfp8(w)
    deq = oq.dequantize_mxfp8(q, s)
    rep = {"format": "mxfp8",
           "granularity": f"e4m3 + e8m0 scale per 32 along K, both operands ({rule} rule)",
           **_weight_fields(w, deq), "bytes": {"before": w.size * element_bytes, "after": q.size + s.size}}
    if x is None:
        return rep
    a = f32(x).reshape(-1, w.shape[1])
    xq, xs = oq.quantize_mxfp8(a, rule)
    a_hat = oq.dequantize_mxfp8(xq, xs)
    out = _output_fields(a.astype(np.float64) @ w.astype(np.float64).T,
                         a_hat.astype(np.float64) @ deq.astype(np.float64).T)
    sat = oq.mxfp8_saturation(a, xs)
    return {**rep, "activations": f"e4m3 + e8m0 per 32 ({rule} rule)",
            "activation_rel_l2": _activation_fields(a, a_hat)["activation_rel_l2"],
            "activation_saturation": {k: sat[k] for k in ("share", "worst_ratio")},
            "output_rel_l2": out["output_rel_l2"], "output_cosine": out["output_cosine"],
            "output_norm_ratio": out["output_norm_ratio"]}


def fp4_saturation(x, scales, outer, fmt="nvfp4") -> dict:
    """quant.py:1260-1297: ratio = block max / (scale * outer) (fp32), saturated above
    6 x (1 + 2^-20)."""
    block = oq.FP4_BLOCKS[fmt]
    a = f32(x).reshape(-1, f32(x).shape[-1])
    rows, k = a.shape
    bmax = np.abs(a.reshape(rows, k // block, block)).max(axis=-1)
    sv = e4m3_to_f32(scales) if fmt == "nvfp4" else oq.e8m0_to_f32(scales)
    step = (sv * f32(outer)[:, None]).astype(F32)
    with np.errstate(**_ERR):
        ratio = np.where(step > 0, (bmax / np.maximum(step, F32(1e-38))).astype(F32), F32(0.0))
    limit = F32(6.0 * (1 + 2.0**-20))
    saturated = int((ratio > limit).sum())
    blocks = rows * (k // block)
    return {"blocks": blocks, "saturated": saturated, "share": _sig(saturated / blocks) if blocks else 0.0,
            "worst_ratio": _sig(float(ratio.max())) if blocks else 0.0}


def fp4_w4a4_error(weight, x, fmt="nvfp4", granularity="token", rotate=None, unbiased=False) -> dict:
    """quant.py:1511-1573 (the weight quantised by :func:`oracle.quant.quantize_fp4`, rotated
    with ``rotate``)."""
    w = f32(weight)
    a = f32(x).reshape(-1, w.shape[1])
    wr = oq.hadamard_rotate(w, rotate) if rotate else w
    rep, (codes, scales, ts) = fp4_error(wr, 4, fmt, unbiased=unbiased)
    a_rot = oq.hadamard_rotate(a, rotate) if rotate else a
    xq, xs, outer = oq.quantize_fp4_activations(a_rot, fmt, granularity)
    sat = fp4_saturation(a_rot, xs, outer, fmt)
    if unbiased:
        outer = (outer * oq.fp4_bias_correction(a_rot, xq, xs, outer, fmt)).astype(F32)
    a_hat = (oq.fp4_values(xq, xs, fmt) * outer[:, None]).astype(F32)
    acc = oq.fp4_values(xq, xs, fmt).astype(np.float64) @ oq.fp4_values(codes, scales, fmt).astype(np.float64).T
    tsv = np.asarray(ts, np.float64).reshape(-1)[None, :]
    new = (acc * (outer.astype(np.float64)[:, None] * tsv)).astype(F32)
    out = _output_fields(a.astype(np.float64) @ w.astype(np.float64).T, new)
    block, kind = oq.FP4_BLOCKS[fmt], "e4m3" if fmt == "nvfp4" else "e8m0"
    rep.update(activations=f"{fmt}: e2m1 + {kind} scale per {block}"
               + (f" x fp32 per {granularity}" if fmt == "nvfp4" else "")
               + (f", Hadamard {rotate}" if rotate else "") + (", unbiased" if unbiased else ""),
               activation_rel_l2=_activation_fields(a_rot, a_hat)["activation_rel_l2"],
               activation_crest=_activation_fields(a, a)["activation_crest"],
               activation_saturation={k: sat[k] for k in ("share", "worst_ratio")}, **out)
    return rep
