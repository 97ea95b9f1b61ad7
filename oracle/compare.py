"""CPU restatement of the reference comparator's element loop and verdict (test
infrastructure only).

Reference: ``src/kernel_agent/kernels/compare.py`` (tolerances and tiers 57-502,
``_non_finite_error`` 565-579, ``_channels`` 582-589, ``_channel_rms`` 592-605,
``_rounding_widening`` 608-628, ``compare_tensors`` 631-790). Element-wise arithmetic is fp32
as torch does it on the CPU (a Python scalar meets an fp32 tensor as an fp32 value); the
norms and the dot product, which torch reduces in its own order, are summed here in float64
and rounded to fp32 once.
"""

from __future__ import annotations

import math

import numpy as np

F32 = np.float32

TOLERANCES = {"f32": (1e-4, 1e-4), "f16": (1e-2, 1e-2), "bf16": (2e-2, 2e-2)}  # 57-61
MAX_MISMATCH = 1e-3  # 63
MAX_OUTLIER = 10.0  # 65
GLOBAL_MIN_NUMEL = 1024  # 67
GLOBAL_TOLERANCES = {"f32": (0.99999, 0.005), "f16": (0.9995, 0.01), "bf16": (0.999, 0.02)}
NEAR_LOSSLESS_BOUNDS = {  # 280-329
    "near-lossless": (0.996, 0.08, 0.02, (0.5, 0.125)),
    "near-lossless-fp4": (0.96, 0.28, 0.04, (1.25, 0.25)),
    "near-lossless-kv": (0.996, 0.08, 0.02, (0.5, 0.125)),
    "relaxed": (0.99, 0.16, 0.04, (0.75, 0.125)),
    "relaxed-fp4": (0.94, 0.36, 0.06, (1.75, 0.25)),
    "relaxed-kv": (0.99, 0.16, 0.04, (0.75, 0.125)),
    "near-lossless-fp4a": (0.96, 0.28, 0.05, (1.5, 0.25)),
    "relaxed-fp4a": (0.94, 0.36, 0.08, (2.0, 0.25)),
}
PERTURBED_BOUNDS = {  # 440-449
    "near-lossless": (0.996, 0.08, 0.03, (0.75, 0.125)),
    "near-lossless-fp4": (0.94, 0.40, 0.12, (2.5, 0.25)),
    "near-lossless-kv": (0.985, 0.16, 0.03, (1.5, 0.125)),
    "relaxed": (0.99, 0.16, 0.06, (1.5, 0.125)),
    "relaxed-fp4": (0.90, 0.55, 0.18, (3.0, 0.25)),
    "relaxed-kv": (0.97, 0.25, 0.06, (2.5, 0.125)),
    "near-lossless-fp4a": (0.90, 0.50, 0.15, (3.0, 0.25)),
    "relaxed-fp4a": (0.85, 0.65, 0.18, (3.5, 0.25)),
}
CHANNEL_MIN_ROWS = 16  # 351
ROUNDING_SPREAD_K = 4.0  # 484
ROUNDING_SPREAD_CAP = 0.125  # 485
ROUNDING_SPREAD_RMS = 2.0  # 486

_ERR = {"over": "ignore", "invalid": "ignore", "divide": "ignore", "under": "ignore"}


def _norm(v: np.ndarray) -> float:
    """``float(t.norm())`` of an fp32 tensor: float64 sum of squares, sqrt, rounded to fp32."""
    return float(F32(math.sqrt(float(np.sum(np.square(v.astype(np.float64)))))))


def _non_finite_error(a: np.ndarray, b: np.ndarray) -> str | None:
    """compare.py:565-579."""
    problems = []
    for label, in_ref, in_new in (
        ("NaN", np.isnan(a), np.isnan(b)),
        ("+inf", a == np.inf, b == np.inf),
        ("-inf", a == -np.inf, b == -np.inf),
    ):
        differ = int((in_ref != in_new).sum())
        if differ:
            problems.append(
                f"{label} at {differ} positions that differ "
                f"(candidate {int(in_new.sum())}, reference {int(in_ref.sum())})"
            )
    return "; ".join(problems) or None


def _channels(ref: np.ndarray) -> np.ndarray | None:
    """compare.py:582-589: per-channel RMS (last dimension), non-finite as 0."""
    if ref.ndim < 2 or ref.size < CHANNEL_MIN_ROWS * ref.shape[-1]:
        return None
    values = np.where(np.isfinite(ref), ref, F32(0)).astype(F32)
    axes = tuple(range(ref.ndim - 1))
    ms = np.mean(np.square(values.astype(np.float64)), axis=axes, keepdims=True)
    return np.sqrt(ms.astype(F32)).astype(F32)


def _channel_rms(ref: np.ndarray, rms: float, floor=None):
    """compare.py:592-605."""
    channel = _channels(ref)
    if floor is not None:
        floor = np.asarray(floor, F32)
        channel = floor if channel is None else np.maximum(channel, floor)
    if channel is None:
        return rms
    return np.broadcast_to(np.maximum(channel, F32(rms)), ref.shape).astype(F32)


def _rounding_widening(ref, rerounded, rms, floor=None):
    """compare.py:608-628."""
    if rerounded is None or rerounded.shape != ref.shape:
        return None
    alt = np.asarray(rerounded, F32)
    with np.errstate(**_ERR):
        diff = np.where(np.isfinite(ref) & np.isfinite(alt), (alt - ref).astype(F32), F32(0))
    spread = float(F32(math.sqrt(float(np.mean(np.square(diff.astype(np.float64))))))) if diff.size else 0.0
    grow = np.asarray(_channel_rms(diff, spread), F32) * F32(ROUNDING_SPREAD_K)
    cap = np.asarray(_channel_rms(ref, rms, floor), F32) * F32(ROUNDING_SPREAD_CAP)
    widen = np.minimum(grow, cap).astype(F32)
    return (widen if widen.ndim else float(widen)), spread


def compare_tensors(name, ref, new, dtype="bf16", tol=None, *, tier="exact", perturbed=False,
                    input_scale=1.0, channel_rms=None, rerounded=None) -> dict:
    """compare.py:631-790 from the dtype checks on: ``ref`` and ``new`` are arrays of the
    same shape holding the tensors' values (``dtype``: "bf16" / "f16" / "f32" for
    floating-point tensors, "int" for integer or boolean ones)."""
    result: dict = {"name": name, "ok": False}
    ref = np.asarray(ref)
    new = np.asarray(new)
    if ref.shape != new.shape:
        result["error"] = f"shape {tuple(new.shape)} != reference {tuple(ref.shape)}"
        return result
    if dtype == "int":
        mismatches = float(F32(np.count_nonzero(ref != new)) / F32(ref.size)) if ref.size else 0.0
        result.update(ok=mismatches == 0, mismatch_frac=mismatches)
        return result
    atol, rtol = tol or TOLERANCES.get(dtype, (1e-3, 1e-3))
    factor = abs(float(input_scale)) or 1.0
    floor = atol * min(1.0, factor)
    atol *= max(1.0, factor)
    full = np.asarray(ref, F32)
    a, b = full, np.asarray(new, F32)
    error = _non_finite_error(a, b)
    if error is not None:
        result["error"] = error
        return result
    finite = np.isfinite(a)
    masked = not bool(finite.all())
    if masked:
        a, b = a[finite], b[finite]
    with np.errstate(**_ERR):
        diff = np.abs(a - b).astype(F32)
        ref_norm, new_norm = _norm(a), _norm(b)
        n = a.size
        signal = n > 0 and ref_norm > floor * math.sqrt(n)
        near = (PERTURBED_BOUNDS if perturbed else NEAR_LOSSLESS_BOUNDS).get(tier)
        allowed = (F32(atol) + (F32(rtol) * np.abs(a)).astype(F32)).astype(F32)
        if perturbed and near is not None and not signal:
            alt_bound = (F32(near[3][0] * atol) + (F32(near[3][1]) * np.abs(a)).astype(F32)).astype(F32)
            allowed = np.maximum(allowed, alt_bound)
        rms = ref_norm / math.sqrt(n) if n else 0.0
        rer = None
        if rerounded is not None and np.shape(rerounded) == full.shape:
            rer = rerounded
        spread = _rounding_widening(full, rer, rms, channel_rms)
        noise = _norm(diff) / math.sqrt(diff.size) if diff.size else 0.0
        widened = False
        if spread is not None:
            widen, total = spread
            ratio = noise / total if total > 0 else (0.0 if noise == 0 else math.inf)
            result.update(rounding_spread=round(total / rms, 6) if rms > 0 else 0.0)
            result.update(error_over_spread=round(ratio, 3))
            if ratio <= ROUNDING_SPREAD_RMS:
                if masked and isinstance(widen, np.ndarray):
                    widen = widen[finite]
                allowed = (allowed + (widen if isinstance(widen, np.ndarray) else F32(widen))).astype(F32)
                widened = True
        count = int(np.count_nonzero(diff > allowed))
        mismatch = float(F32(count) / F32(n)) if n else 0.0
        outlier = float((diff / np.maximum(allowed, F32(1e-30))).astype(F32).max()) if n else 0.0
        denom = ref_norm * new_norm
        dot = F32(float(np.dot(a.ravel().astype(np.float64), b.ravel().astype(np.float64))))
        cos = float(F32(dot / F32(denom))) if denom > 0 else 1.0
        rel_l2 = _norm(diff) / ref_norm if ref_norm > 0 else 0.0
    result.update(
        max_abs_err=float(diff.max()) if diff.size else 0.0,
        mean_abs_err=float(F32(np.mean(diff.astype(np.float64)))) if diff.size else 0.0,
        mismatch_frac=round(mismatch, 6),
        max_err_ratio=round(outlier, 3),
        cosine=round(cos, 7),
        rel_l2=float(f"{rel_l2:.4g}"),
        atol=atol,
        rtol=rtol,
    )
    problems = []
    min_cos, max_rel = GLOBAL_TOLERANCES.get(dtype, GLOBAL_TOLERANCES["f32"])
    if near is not None and signal:
        min_cos, max_rel, max_norm_change, (e_atol, e_rtol) = near
        scale = rms
        if perturbed:
            scale = _channel_rms(full, rms, channel_rms)
            if masked and isinstance(scale, np.ndarray):
                scale = scale[finite]
        with np.errstate(**_ERR):
            if isinstance(scale, np.ndarray):
                first = (F32(e_atol) * scale).astype(F32)
            else:
                first = F32(e_atol * scale)
            den = (first + (F32(e_rtol) * np.abs(a)).astype(F32)).astype(F32)
            element = float((diff / den).astype(F32).max())
        norm_ratio = new_norm / ref_norm
        result.update(
            tier=tier,
            max_err_over_rms=round(float(diff.max()) / rms, 4),
            element_ratio=round(element, 4),
            norm_ratio=round(norm_ratio, 6),
        )
        if element > 1.0:
            where = " on redrawn inputs" if perturbed else ""
            of = " (the larger of the tensor's and its channel's)" if perturbed else ""
            problems.append(
                f"an element is {element:.3g}x its {tier} tolerance away{where} "
                f"({e_atol:g} x RMS{of} + {e_rtol:g} x |reference|)"
            )
        if abs(norm_ratio - 1.0) > max_norm_change:
            problems.append(
                f"norm x{norm_ratio:.4f} (allowed ±{max_norm_change:.0%}): "
                "a systematic error, not rounding noise"
            )
        whole = True
    else:
        tolerance = "tolerance"
        if widened:
            tolerance += (
                f" (with {ROUNDING_SPREAD_K:g} x the reference's own rounding spread, "
                f"{result['rounding_spread']:.3%} of its RMS)"
            )
        elif spread is not None:
            tolerance += (
                f" (the error's RMS is {result['error_over_spread']:.3g} x the reference's own "
                f"rounding spread, more than {ROUNDING_SPREAD_RMS:g} x: not rounding)"
            )
        if mismatch > MAX_MISMATCH:
            problems.append(f"{mismatch:.4%} of elements outside {tolerance} (max {MAX_MISMATCH:.2%})")
        if outlier > MAX_OUTLIER:
            problems.append(
                f"an element is {outlier:.3g}x its {tolerance} away (max {MAX_OUTLIER:g}x per element)"
            )
        whole = n > GLOBAL_MIN_NUMEL and signal
    if whole:
        if cos < min_cos:
            problems.append(f"cosine {cos:.6f} < {min_cos}")
        if rel_l2 > max_rel:
            problems.append(f"relative L2 error {rel_l2:.4g} > {max_rel}")
    if problems:
        result["error"] = "; ".join(problems)
    result["ok"] = not problems
    return result
