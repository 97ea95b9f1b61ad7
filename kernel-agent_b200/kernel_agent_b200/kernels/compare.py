"""GPU drop-in for ``kernel_agent.kernels.compare`` (kernel-agent 0.1.0,
``src/kernel_agent/kernels/compare.py``): the evaluator's comparator with the same
constants, tiers, functions, result dictionaries and error messages.

The element loop of :func:`compare_tensors` (compare.py:684-739: the non-finite positions,
``diff > atol + rtol·|ref|``, the largest ``diff / allowed``, the norms and the dot product,
the reduced tiers' element ratio) is one fused reduction in ``libkab.so`` (``kab_compare``):
one read of ``ref`` and ``new`` for the exact tier, a second (L2-resident for outputs that
fit in L2) for the reduced tiers, whose element bound needs the tensor's RMS first. Counts
and maxima use the reference's fp32 roundings and are bit for bit torch's; the norms and the
dot product are float64 sums (torch sums them in fp32 in its own order, so cosine / relative
L2 / norm ratio can differ from the CPU reference in the last reported digit). The verdict
logic (compare.py:740-790) runs on the host on those numbers, as the reference's does.

The routing around it (:func:`compare_structures`, :func:`compare_output`,
:func:`compare_grown`, :func:`compare_written`, :func:`compare_side_effects`) follows the
reference's rules; their masks and slices are torch operations on the GPU, and every
tensor comparison goes through :func:`compare_tensors`.
"""

from __future__ import annotations

import ctypes
import dataclasses
import math
from typing import Any

import numpy as np
import torch

from .. import _native as nat

# ------------------------------------------------------------------ constants (compare.py:57-502)

TOLERANCES: dict[torch.dtype, tuple[float, float]] = {
    torch.float32: (1e-4, 1e-4),
    torch.float16: (1e-2, 1e-2),
    torch.bfloat16: (2e-2, 2e-2),
}
MAX_MISMATCH = 1e-3
MAX_OUTLIER = 10.0
GLOBAL_MIN_NUMEL = 1024
GLOBAL_TOLERANCES: dict[torch.dtype, tuple[float, float]] = {
    torch.float32: (0.99999, 0.005),
    torch.float16: (0.9995, 0.01),
    torch.bfloat16: (0.999, 0.02),
}
EXACT_TIER = "exact"
NEAR_LOSSLESS_TIER = "near-lossless"
NEAR_LOSSLESS_FP4_TIER = "near-lossless-fp4"
NEAR_LOSSLESS_KV_TIER = "near-lossless-kv"
RELAXED_TIER = "relaxed"
RELAXED_FP4_TIER = "relaxed-fp4"
RELAXED_KV_TIER = "relaxed-kv"
NEAR_LOSSLESS_FP4A_TIER = "near-lossless-fp4a"
RELAXED_FP4A_TIER = "relaxed-fp4a"
TIERS = (
    EXACT_TIER, NEAR_LOSSLESS_TIER, NEAR_LOSSLESS_FP4_TIER, NEAR_LOSSLESS_KV_TIER, RELAXED_TIER,
    RELAXED_FP4_TIER, RELAXED_KV_TIER, NEAR_LOSSLESS_FP4A_TIER, RELAXED_FP4A_TIER,
)
QUALITIES = (EXACT_TIER, NEAR_LOSSLESS_TIER, RELAXED_TIER)
REDUCED_QUALITIES = (NEAR_LOSSLESS_TIER, RELAXED_TIER)
DEFAULT_QUALITY = RELAXED_TIER
REDUCED_PRECISIONS = (
    "fp8_weights", "reduced", "fp4_weights", "fp8_w8a8", "fp8_mx", "fp8_kv", "int8_weights",
    "int8_w8a8", "fp4_w4a4",
)
PRECISION_TIERS = {
    "fp4_weights": NEAR_LOSSLESS_FP4_TIER,
    "fp8_kv": NEAR_LOSSLESS_KV_TIER,
    "fp4_w4a4": NEAR_LOSSLESS_FP4A_TIER,
}
RELAXED_PRECISION_TIERS = {
    "fp4_weights": RELAXED_FP4_TIER,
    "fp8_kv": RELAXED_KV_TIER,
    "fp4_w4a4": RELAXED_FP4A_TIER,
}
QUALITY_TIERS: dict[str, tuple[str, dict[str, str]]] = {
    NEAR_LOSSLESS_TIER: (NEAR_LOSSLESS_TIER, PRECISION_TIERS),
    RELAXED_TIER: (RELAXED_TIER, RELAXED_PRECISION_TIERS),
}
PRECISIONS = (EXACT_TIER, *REDUCED_PRECISIONS)
NEAR_LOSSLESS_MIN_COSINE = 0.996
NEAR_LOSSLESS_MAX_REL_L2 = 0.08
NEAR_LOSSLESS_MAX_NORM_CHANGE = 0.02
NEAR_LOSSLESS_ELEMENT = (0.5, 0.125)
NEAR_LOSSLESS_FP4_MIN_COSINE = 0.96
NEAR_LOSSLESS_FP4_MAX_REL_L2 = 0.28
NEAR_LOSSLESS_FP4_MAX_NORM_CHANGE = 0.04
NEAR_LOSSLESS_FP4_ELEMENT = (1.25, 0.25)
RELAXED_MIN_COSINE = 0.99
RELAXED_MAX_REL_L2 = 0.16
RELAXED_MAX_NORM_CHANGE = 0.04
RELAXED_ELEMENT = (0.75, 0.125)
RELAXED_FP4_MIN_COSINE = 0.94
RELAXED_FP4_MAX_REL_L2 = 0.36
RELAXED_FP4_MAX_NORM_CHANGE = 0.06
RELAXED_FP4_ELEMENT = (1.75, 0.25)
NEAR_LOSSLESS_FP4A_MIN_COSINE = 0.96
NEAR_LOSSLESS_FP4A_MAX_REL_L2 = 0.28
NEAR_LOSSLESS_FP4A_MAX_NORM_CHANGE = 0.05
NEAR_LOSSLESS_FP4A_ELEMENT = (1.5, 0.25)
RELAXED_FP4A_MIN_COSINE = 0.94
RELAXED_FP4A_MAX_REL_L2 = 0.36
RELAXED_FP4A_MAX_NORM_CHANGE = 0.08
RELAXED_FP4A_ELEMENT = (2.0, 0.25)


def _bounds(cos, rel, norm, element):
    return (cos, rel, norm, element)


NEAR_LOSSLESS_BOUNDS: dict[str, tuple[float, float, float, tuple[float, float]]] = {
    NEAR_LOSSLESS_TIER: _bounds(NEAR_LOSSLESS_MIN_COSINE, NEAR_LOSSLESS_MAX_REL_L2,
                                NEAR_LOSSLESS_MAX_NORM_CHANGE, NEAR_LOSSLESS_ELEMENT),
    NEAR_LOSSLESS_FP4_TIER: _bounds(NEAR_LOSSLESS_FP4_MIN_COSINE, NEAR_LOSSLESS_FP4_MAX_REL_L2,
                                    NEAR_LOSSLESS_FP4_MAX_NORM_CHANGE, NEAR_LOSSLESS_FP4_ELEMENT),
    NEAR_LOSSLESS_KV_TIER: _bounds(NEAR_LOSSLESS_MIN_COSINE, NEAR_LOSSLESS_MAX_REL_L2,
                                   NEAR_LOSSLESS_MAX_NORM_CHANGE, NEAR_LOSSLESS_ELEMENT),
    RELAXED_TIER: _bounds(RELAXED_MIN_COSINE, RELAXED_MAX_REL_L2, RELAXED_MAX_NORM_CHANGE,
                          RELAXED_ELEMENT),
    RELAXED_FP4_TIER: _bounds(RELAXED_FP4_MIN_COSINE, RELAXED_FP4_MAX_REL_L2,
                              RELAXED_FP4_MAX_NORM_CHANGE, RELAXED_FP4_ELEMENT),
    RELAXED_KV_TIER: _bounds(RELAXED_MIN_COSINE, RELAXED_MAX_REL_L2, RELAXED_MAX_NORM_CHANGE,
                             RELAXED_ELEMENT),
    NEAR_LOSSLESS_FP4A_TIER: _bounds(NEAR_LOSSLESS_FP4A_MIN_COSINE, NEAR_LOSSLESS_FP4A_MAX_REL_L2,
                                     NEAR_LOSSLESS_FP4A_MAX_NORM_CHANGE, NEAR_LOSSLESS_FP4A_ELEMENT),
    RELAXED_FP4A_TIER: _bounds(RELAXED_FP4A_MIN_COSINE, RELAXED_FP4A_MAX_REL_L2,
                               RELAXED_FP4A_MAX_NORM_CHANGE, RELAXED_FP4A_ELEMENT),
}
CHANNEL_MIN_ROWS = 16
PERTURBED_BOUNDS: dict[str, tuple[float, float, float, tuple[float, float]]] = {
    NEAR_LOSSLESS_TIER: (0.996, 0.08, 0.03, (0.75, 0.125)),
    NEAR_LOSSLESS_FP4_TIER: (0.94, 0.40, 0.12, (2.5, 0.25)),
    NEAR_LOSSLESS_KV_TIER: (0.985, 0.16, 0.03, (1.5, 0.125)),
    RELAXED_TIER: (0.99, 0.16, 0.06, (1.5, 0.125)),
    RELAXED_FP4_TIER: (0.90, 0.55, 0.18, (3.0, 0.25)),
    RELAXED_KV_TIER: (0.97, 0.25, 0.06, (2.5, 0.125)),
    NEAR_LOSSLESS_FP4A_TIER: (0.90, 0.50, 0.15, (3.0, 0.25)),
    RELAXED_FP4A_TIER: (0.85, 0.65, 0.18, (3.5, 0.25)),
}
ROUNDING_SPREAD_K = 4.0
ROUNDING_SPREAD_CAP = 0.125
ROUNDING_SPREAD_RMS = 2.0
WRITTEN_MAX_FRACTION = 0.5
WRITTEN_MIN_DENSITY = 0.75
#: The tier of this process's comparisons when a call passes none (compare.py:502); the
#: evaluator sets it from the capture.
TIER = EXACT_TIER
_PLAIN = (torch.Tensor, torch.nn.Parameter)
_F32 = np.float32


def tier_of(capture: dict[str, Any] | None) -> str:
    """compare.py:506-509."""
    name = (capture or {}).get("tier")
    return name if name in TIERS else EXACT_TIER


def tier_for(quality: str | None, precision: str | None) -> str:
    """compare.py:512-521."""
    if quality not in QUALITY_TIERS or precision not in REDUCED_PRECISIONS:
        return EXACT_TIER
    main, own = QUALITY_TIERS[str(quality)]
    return own.get(str(precision), main)


def allows_reduced(quality: str | None) -> bool:
    """compare.py:524-527."""
    return quality in REDUCED_QUALITIES


def flatten(value: Any, prefix: str = "out", depth: int = 0) -> dict[str, torch.Tensor]:
    """compare.py:530-550: nested containers / dataclasses / objects into named tensors."""
    found: dict[str, torch.Tensor] = {}
    if depth > 6 or value is None:
        return found
    if isinstance(value, torch.Tensor):
        found[prefix] = value
    elif isinstance(value, dict):
        for key, item in value.items():
            found.update(flatten(item, f"{prefix}.{key}", depth + 1))
    elif isinstance(value, tuple | list):
        for i, item in enumerate(value):
            found.update(flatten(item, f"{prefix}[{i}]", depth + 1))
    elif dataclasses.is_dataclass(value) and not isinstance(value, type):
        for f in dataclasses.fields(value):
            found.update(flatten(getattr(value, f.name, None), f"{prefix}.{f.name}", depth + 1))
    elif hasattr(value, "__dict__") and not isinstance(value, torch.nn.Module):
        for key, item in vars(value).items():
            if not key.startswith("__"):
                found.update(flatten(item, f"{prefix}.{key}", depth + 1))
    return found


def type_error(new: Any) -> str | None:
    """compare.py:553-562."""
    if type(new) in _PLAIN:
        return None
    if isinstance(new, torch.Tensor):
        return (
            f"got a {type(new).__name__} (a torch.Tensor subclass); return plain tensors "
            "(a subclass can defer the computation until the result is read)"
        )
    return f"expected tensor, got {type(new).__name__}"


# ------------------------------------------------------------------ the fused element loop


class _Pass:
    """One ``kab_compare`` launch and its result on the host."""

    def __init__(self, ref: torch.Tensor, new: torch.Tensor, rer: torch.Tensor | None, *,
                 atol: float, rtol: float, channels: int, alt=None, widen=None, element=None):
        n = ref.numel()
        p = nat.KabCompareParams()
        p.ref, p.new_ = ref.data_ptr(), new.data_ptr()
        p.rerounded = rer.data_ptr() if rer is not None else None
        p.n, p.channels = n, channels
        p.dtype = nat.dtype_code(ref)
        p.has_rerounded = int(rer is not None)
        p.vector = int(all(t is None or t.data_ptr() % 16 == 0 for t in (ref, new, rer))
                       and ref.element_size() in (2, 4))
        p.atol, p.rtol = float(_F32(atol)), float(_F32(rtol))
        if alt is not None:
            p.alt_bound, p.alt_atol, p.alt_rtol = 1, float(_F32(alt[0])), float(_F32(alt[1]))
        self._keep = []
        if widen is not None:
            if isinstance(widen, torch.Tensor):
                w = widen.float().contiguous()
                self._keep.append(w)
                p.widen_mode, p.widen_channel = 2, w.data_ptr()
            else:
                p.widen_mode, p.widen_scalar = 1, float(_F32(widen))
        if element is not None:
            first_or_scale, e_atol, e_rtol = element
            p.element_rtol = float(_F32(e_rtol))
            if isinstance(first_or_scale, torch.Tensor):
                sc = first_or_scale.float().contiguous()
                self._keep.append(sc)
                p.element_mode, p.element_scale, p.element_atol = 2, sc.data_ptr(), float(_F32(e_atol))
            else:
                p.element_mode, p.element_first = 1, float(_F32(first_or_scale))
        stream = nat.stream_of(ref)
        nbytes = int(nat.query("kab_compare_scratch_bytes", n))
        scratch = torch.empty(max(nbytes, 16), dtype=torch.uint8, device=ref.device)
        out = torch.empty(ctypes.sizeof(nat.KabCompareResult), dtype=torch.uint8, device=ref.device)
        nat.call("kab_compare", ctypes.byref(p), scratch.data_ptr(), scratch.numel(), out.data_ptr(), stream)
        host = out.cpu()  # one device-to-host read (the reference's .item() calls)
        res = nat.KabCompareResult.from_buffer_copy(bytes(host.numpy().tobytes()))
        self.count = list(res.count)
        self.sum = list(res.sum)
        self.max = list(res.max)


def _channel_rms_of(x: torch.Tensor, alt: torch.Tensor | None = None) -> torch.Tensor | None:
    """compare.py:582-589 ``_channels`` on the GPU (``alt``: of ``alt - x``, compare.py:622-625):
    per-channel RMS ``[C]`` (fp32), None for fewer than CHANNEL_MIN_ROWS rows."""
    if x.dim() < 2 or x.numel() < CHANNEL_MIN_ROWS * x.shape[-1]:
        return None
    c = x.shape[-1]
    rows = x.numel() // c
    rms = torch.empty(c, dtype=torch.float32, device=x.device)
    nbytes = int(nat.query("kab_channel_rms_scratch_bytes", rows, c))
    scratch = torch.empty(max(nbytes, 16), dtype=torch.uint8, device=x.device)
    nat.call("kab_channel_rms", x.data_ptr(), nat.ptr(alt), nat.dtype_code(x), rows, c, rms.data_ptr(),
             scratch.data_ptr(), scratch.numel(), nat.stream_of(x))
    return rms


def _per_channel(ref: torch.Tensor, rms: float, floor: torch.Tensor | None, alt=None):
    """compare.py:592-605 ``_channel_rms`` as a per-channel vector ``[C]`` or the scalar."""
    channel = _channel_rms_of(ref, alt)
    if floor is not None:
        fl = floor.to(ref.device, torch.float32).reshape(-1)
        if fl.numel() not in (1, ref.shape[-1]):
            raise ValueError("channel_rms must broadcast along the last dimension")
        fl = fl.expand(ref.shape[-1]) if fl.numel() == 1 else fl
        channel = fl if channel is None else torch.maximum(channel, fl)
    if channel is None:
        return rms
    return channel.clamp_min(rms)


def _operands(ref: torch.Tensor, new: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """``ref`` on ``new``'s device, both contiguous in a dtype the kernel reads (others as
    fp32, the reference's ``.float()``)."""
    a = ref.detach().to(new.device)
    b = new.detach()
    if a.dtype not in nat.DTYPES:
        a, b = a.float(), b.float()
    return a.contiguous(), b.contiguous()


def compare_tensors(
    name: str,
    ref: torch.Tensor,
    new: torch.Tensor,
    tol: tuple[float, float] | None = None,
    *,
    tier: str | None = None,
    perturbed: bool = False,
    input_scale: float = 1.0,
    channel_rms: torch.Tensor | None = None,
    rerounded: torch.Tensor | None = None,
) -> dict[str, Any]:
    """compare.py:631-790: one tensor against its reference (tier, perturbed bounds, input
    scale, channel RMS floor and rounding spread as there), on the GPU."""
    result: dict[str, Any] = {"name": name, "ok": False}
    error = type_error(new)
    if error is not None:
        result["error"] = error
        return result
    if ref.shape != new.shape:
        result["error"] = f"shape {tuple(new.shape)} != reference {tuple(ref.shape)}"
        return result
    if ref.dtype != new.dtype:
        result["error"] = f"dtype {new.dtype} != reference {ref.dtype}"
        return result
    if new.layout != ref.layout or new.device.type != ref.device.type:
        result["error"] = (
            f"{new.layout} tensor on {new.device.type} != reference "
            f"{ref.layout} tensor on {ref.device.type}"
        )
        return result
    nat.require_cuda(new)
    if not ref.is_floating_point():
        if ref.numel():
            differ = int(torch.count_nonzero(ref.to(new.device) != new))
            mismatches = float(_F32(differ) / _F32(ref.numel()))
        else:
            mismatches = 0.0
        result.update(ok=mismatches == 0, mismatch_frac=mismatches)
        return result
    atol, rtol = tol or TOLERANCES.get(ref.dtype, (1e-3, 1e-3))
    factor = abs(float(input_scale)) or 1.0
    floor = atol * min(1.0, factor)
    atol *= max(1.0, factor)
    a, b = _operands(ref, new)
    alt = _like(rerounded, ref)
    alt_t = None if alt is None else alt.to(new.device).to(a.dtype).contiguous()
    channels = a.shape[-1] if a.dim() >= 1 and a.numel() else 1
    first = _Pass(a, b, alt_t, atol=atol, rtol=rtol, channels=channels)
    c = first.count
    problems_nf = []
    for label, kr, kn, kd in (("NaN", 0, 1, 2), ("+inf", 3, 4, 5), ("-inf", 6, 7, 8)):
        if c[kd]:
            problems_nf.append(f"{label} at {c[kd]} positions that differ (candidate {c[kn]}, reference {c[kr]})")
    if problems_nf:
        result["error"] = "; ".join(problems_nf)
        return result
    n = c[nat.CMP_NCOUNT - 2]  # finite elements of ref
    total = a.numel()
    masked = n < total
    s = first.sum
    ref_norm = float(_F32(math.sqrt(s[0])))
    new_norm = float(_F32(math.sqrt(s[1])))
    signal = n > 0 and ref_norm > floor * math.sqrt(n)
    near = (PERTURBED_BOUNDS if perturbed else NEAR_LOSSLESS_BOUNDS).get(tier or TIER)
    alt_bound = None
    if perturbed and near is not None and not signal:
        alt_bound = (near[3][0] * atol, near[3][1])
    rms = ref_norm / math.sqrt(n) if n else 0.0
    diff_norm = float(_F32(math.sqrt(s[3])))
    noise = diff_norm / math.sqrt(n) if n else 0.0
    widen = None
    widened = False
    if alt_t is not None:  # compare.py:608-628, 702-714
        spread = float(_F32(math.sqrt(s[5] / total))) if total else 0.0
        grow = _per_channel(a, spread, None, alt=alt_t)
        cap = _per_channel(a, rms, channel_rms)
        grow = grow * _F32(ROUNDING_SPREAD_K) if isinstance(grow, torch.Tensor) else float(_F32(spread) * _F32(ROUNDING_SPREAD_K))
        cap = cap * _F32(ROUNDING_SPREAD_CAP) if isinstance(cap, torch.Tensor) else float(_F32(cap) * _F32(ROUNDING_SPREAD_CAP))
        if isinstance(grow, torch.Tensor) or isinstance(cap, torch.Tensor):
            g_t = grow if isinstance(grow, torch.Tensor) else torch.full((channels,), grow, device=a.device)
            c_t = cap if isinstance(cap, torch.Tensor) else torch.full((channels,), cap, device=a.device)
            widen_v: Any = torch.minimum(g_t, c_t)
        else:
            widen_v = min(grow, cap)
        ratio = noise / spread if spread > 0 else (0.0 if noise == 0 else math.inf)
        result.update(rounding_spread=round(spread / rms, 6) if rms > 0 else 0.0)
        result.update(error_over_spread=round(ratio, 3))
        if ratio <= ROUNDING_SPREAD_RMS:
            widen, widened = widen_v, True
    element_spec = None
    if near is not None and signal:
        e_atol, e_rtol = near[3]
        if perturbed:
            scale = _per_channel(a, rms, channel_rms)
        else:
            scale = rms
        if isinstance(scale, torch.Tensor):
            element_spec = (scale, e_atol, e_rtol)
        else:
            element_spec = (e_atol * scale, e_atol, e_rtol)
    second = first
    if alt_bound is not None or widen is not None or element_spec is not None:
        second = _Pass(a, b, None, atol=atol, rtol=rtol, channels=channels, alt=alt_bound,
                       widen=widen, element=element_spec)
    mismatch = float(_F32(second.count[nat.CMP_NCOUNT - 1]) / _F32(n)) if n else 0.0
    outlier = float(second.max[1]) if n else 0.0
    denom = ref_norm * new_norm
    dot = _F32(s[2])
    cos = float(_F32(dot / _F32(denom))) if denom > 0 else 1.0
    rel_l2 = diff_norm / ref_norm if ref_norm > 0 else 0.0
    result.update(
        max_abs_err=float(first.max[0]) if n else 0.0,
        mean_abs_err=float(_F32(s[4] / n)) if n else 0.0,
        mismatch_frac=round(mismatch, 6),
        max_err_ratio=round(outlier, 3),
        cosine=round(cos, 7),
        rel_l2=float(f"{rel_l2:.4g}"),
        atol=atol,
        rtol=rtol,
    )
    problems = []
    min_cos, max_rel = GLOBAL_TOLERANCES.get(ref.dtype, GLOBAL_TOLERANCES[torch.float32])
    if near is not None and signal:
        min_cos, max_rel, max_norm_change, (e_atol, e_rtol) = near
        element = float(second.max[2])
        norm_ratio = new_norm / ref_norm
        result.update(
            tier=tier or TIER,
            max_err_over_rms=round(float(first.max[0]) / rms, 4),
            element_ratio=round(element, 4),
            norm_ratio=round(norm_ratio, 6),
        )
        if element > 1.0:
            where = " on redrawn inputs" if perturbed else ""
            of = " (the larger of the tensor's and its channel's)" if perturbed else ""
            problems.append(
                f"an element is {element:.3g}x its {tier or TIER} tolerance away{where} "
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
        elif alt_t is not None:
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


def _like(rerounded: Any, ref: torch.Tensor) -> torch.Tensor | None:
    """compare.py:793-803."""
    if (
        not isinstance(rerounded, torch.Tensor)
        or type_error(rerounded) is not None
        or rerounded.shape != ref.shape
        or rerounded.dtype != ref.dtype
    ):
        return None
    return rerounded.detach()


# ------------------------------------------------------------------ caches and structures


def grown_dim(before: Any, after: Any) -> int | None:
    """compare.py:806-825: the dimension along which ``after`` is ``before`` grown."""
    if not (isinstance(before, torch.Tensor) and isinstance(after, torch.Tensor)):
        return None
    if (
        not before.is_floating_point()
        or before.dtype != after.dtype
        or before.dim() != after.dim()
        or before.layout != torch.strided
        or after.layout != torch.strided
        or before.numel() == 0
    ):
        return None
    dims = [d for d in range(before.dim()) if before.shape[d] != after.shape[d]]
    if len(dims) != 1 or after.shape[dims[0]] < before.shape[dims[0]]:
        return None
    return dims[0]


def _same(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """Elementwise equality with NaN equal to NaN."""
    return (a == b) | (torch.isnan(a) & torch.isnan(b))


def _mismatched(new, ref) -> bool:
    return (
        type_error(new) is not None
        or new.shape != ref.shape
        or new.dtype != ref.dtype
        or new.layout != ref.layout
        or new.device.type != ref.device.type
    )


def compare_grown(name, before, ref, new, dim, *, tier=None, perturbed=False, input_scale=1.0,
                  rerounded=None) -> dict[str, Any]:
    """compare.py:833-915: a cache grown along ``dim``: the appended rows with the tier's
    checks, the kept part bit for bit where the reference kept it."""
    kw: dict[str, Any] = {"tier": tier, "perturbed": perturbed, "input_scale": input_scale}
    if _mismatched(new, ref):
        return compare_tensors(name, ref, new, rerounded=rerounded, **kw)
    alt = _like(rerounded, ref)
    kept, total = before.shape[dim], ref.shape[dim]
    ref, before = ref.detach().to(new.device), before.detach().to(new.device)
    new = new.detach()
    appended = total - kept
    channels = _channel_rms_of(ref.float().contiguous()) if perturbed else None
    if channels is not None:
        shape = [1] * ref.dim()
        shape[-1] = ref.shape[-1]
        channels = channels.reshape(shape)
        if dim == ref.dim() - 1:
            channels = channels.narrow(dim, kept, appended)
    result = compare_tensors(
        name, ref.narrow(dim, kept, appended), new.narrow(dim, kept, appended),
        channel_rms=channels,
        rerounded=None if alt is None else alt.to(new.device).narrow(dim, kept, appended), **kw,
    )
    result["grown"] = {"dim": dim, "kept": kept, "appended": appended}
    rows = f"{appended} appended row{'s' if appended != 1 else ''} along dim {dim}"
    problems = [f"the {rows} (after {kept} kept): {result['error']}"] if "error" in result else []
    ref_old, new_old = ref.narrow(dim, 0, kept), new.narrow(dim, 0, kept)
    unchanged = _same(ref_old, before)
    if bool(unchanged.all()):
        moved = int((~_same(new_old, before)).sum())
        result["kept_changed"] = moved
        if moved:
            problems.append(
                f"{moved} of the {before.numel()} elements of the {kept} kept rows along dim "
                f"{dim} changed; the reference keeps them as they were (it only appends)"
            )
    else:
        changed = ~unchanged | ~_same(new_old, before)
        count = int(changed.sum())
        old_alt = None if alt is None else alt.to(new.device).narrow(dim, 0, kept)[changed]
        old = compare_tensors(name, ref_old[changed], new_old[changed], rerounded=old_alt, **kw)
        result["changed_elements"] = count
        if not old["ok"]:
            problems.append(f"the {count} changed elements of the {kept} kept rows: {old['error']}")
    result.pop("error", None)
    if problems:
        result["error"] = "; ".join(problems)
    result["ok"] = not problems
    return result


def written_box(before: Any, after: Any) -> list[torch.Tensor] | None:
    """compare.py:918-953: the indices per dimension of rows a call wrote into ``before``."""
    if not (isinstance(before, torch.Tensor) and isinstance(after, torch.Tensor)):
        return None
    if (
        not before.is_floating_point()
        or before.dtype != after.dtype
        or before.shape != after.shape
        or before.layout != torch.strided
        or after.layout != torch.strided
        or before.dim() == 0
        or before.numel() == 0
    ):
        return None
    changed = ~_same(after.detach(), before.detach().to(after.device))
    count = int(changed.sum())
    if count == 0:
        return None
    hits = [changed.movedim(d, 0).reshape(n, -1).any(1) for d, n in enumerate(changed.shape)]
    sizes = [int(h.sum()) for h in hits]
    box = math.prod(sizes)
    if (
        box > WRITTEN_MAX_FRACTION * changed.numel()
        or count < WRITTEN_MIN_DENSITY * box
        or not any(s == n > 1 for s, n in zip(sizes, changed.shape, strict=True))
    ):
        return None
    return [h.nonzero().flatten() for h in hits]


def compare_written(name, before, ref, new, box, *, tier=None, perturbed=False, input_scale=1.0,
                    rerounded=None) -> dict[str, Any]:
    """compare.py:956-1034: rows written into an input: the box with the tier's checks, the
    rest bit for bit."""
    kw: dict[str, Any] = {"tier": tier, "perturbed": perturbed, "input_scale": input_scale}
    if _mismatched(new, ref):
        return compare_tensors(name, ref, new, rerounded=rerounded, **kw)
    alt = _like(rerounded, ref)
    ref, before = ref.detach().to(new.device), before.detach().to(new.device)
    new = new.detach()
    box = [index.to(new.device) for index in box]

    def part(t: torch.Tensor) -> torch.Tensor:
        for d, index in enumerate(box):
            if index.numel() < t.shape[d]:
                t = t.index_select(d, index)
        return t

    channels = _channel_rms_of(ref.float().contiguous()) if perturbed else None
    if channels is not None:
        if box[-1].numel() < ref.shape[-1]:
            channels = channels.index_select(0, box[-1])
        shape = [1] * ref.dim()
        shape[-1] = channels.numel()
        channels = channels.reshape(shape)
    result = compare_tensors(
        name, part(ref), part(new), channel_rms=channels,
        rerounded=None if alt is None else part(alt.to(new.device)), **kw,
    )
    sizes = [int(index.numel()) for index in box]
    result["written"] = {"box": sizes, "of": list(ref.shape)}
    written = f"written {sizes} of {list(ref.shape)}"
    where = f"the {written} (where the reference changed the input)"
    problems = [f"{where}: {result['error']}"] if "error" in result else []
    inside = torch.ones((), dtype=torch.bool, device=new.device)
    for d, index in enumerate(box):
        hit = torch.zeros(ref.shape[d], dtype=torch.bool, device=new.device)
        hit[index] = True
        inside = inside & hit.view([-1 if i == d else 1 for i in range(ref.dim())])
    moved = int((~_same(new, before) & ~inside).sum())
    result["kept_changed"] = moved
    if moved:
        problems.append(
            f"{moved} of the {ref.numel() - math.prod(sizes)} elements outside the {written} "
            "changed; the reference keeps them as they were (it only writes the box)"
        )
    result.pop("error", None)
    if problems:
        result["error"] = "; ".join(problems)
    result["ok"] = not problems
    return result


def compare_output(name, ref, new, inputs=(), *, tier=None, perturbed=False, input_scale=1.0,
                   rerounded=None) -> dict[str, Any]:
    """compare.py:1037-1071: grown cache, written cache, or a plain tensor comparison."""
    kw: dict[str, Any] = {"tier": tier, "perturbed": perturbed, "input_scale": input_scale,
                          "rerounded": rerounded}
    for before in inputs:
        dim = grown_dim(before, ref)
        if dim is None:
            continue
        lead = ref.detach().narrow(dim, 0, before.shape[dim])
        if bool(_same(lead, before.detach().to(lead.device)).all()):
            return compare_grown(name, before, ref, new, dim, **kw)
    for before in inputs:
        box = written_box(before, ref)
        if box is not None:
            return compare_written(name, before, ref, new, box, **kw)
    return compare_tensors(name, ref, new, **kw)


def compare_structures(ref, new, prefix: str = "out", *, inputs=None, tier=None, perturbed=False,
                       input_scale=1.0, rerounded=None) -> list[dict[str, Any]]:
    """compare.py:1074-1103: the candidate's output against the reference's, tensor by tensor."""
    ref_flat = flatten(ref, prefix)
    new_flat = flatten(new, prefix)
    alt_flat = flatten(rerounded, prefix)
    sources = list(flatten(inputs, "in").values())
    kw: dict[str, Any] = {"tier": tier, "perturbed": perturbed, "input_scale": input_scale}
    results = []
    for name, tensor in ref_flat.items():
        if name not in new_flat:
            results.append({"name": name, "ok": False, "error": "missing in candidate output"})
            continue
        results.append(compare_output(name, tensor, new_flat[name], sources,
                                      rerounded=alt_flat.get(name), **kw))
    return results


def compare_side_effects(pre, ref_post, new_post, prefix: str = "args", *, tier=None,
                         perturbed=False, input_scale=1.0, rerounded=None) -> list[dict[str, Any]]:
    """compare.py:1106-1137: the post-call state of a call's arguments."""
    return compare_side_effects_flat(
        flatten(pre, prefix), flatten(ref_post, prefix), flatten(new_post, prefix), tier=tier,
        perturbed=perturbed, input_scale=input_scale, rerounded_flat=flatten(rerounded, prefix),
    )


def compare_side_effects_flat(pre_flat, ref_flat, new_flat, *, tier=None, perturbed=False,
                              input_scale=1.0, rerounded_flat=None) -> list[dict[str, Any]]:
    """compare.py:1140-1182: in-place updates compared on the elements either side changed."""
    kw: dict[str, Any] = {"tier": tier, "perturbed": perturbed, "input_scale": input_scale}
    results: list[dict[str, Any]] = []
    for name, ref in ref_flat.items():
        new = new_flat.get(name)
        if new is None:
            results.append({"name": name, "ok": False, "error": "missing in candidate arguments"})
            continue
        alt = (rerounded_flat or {}).get(name)
        before = pre_flat.get(name)
        if before is not None and (dim := grown_dim(before, ref)) is not None:
            results.append(compare_grown(name, before, ref, new, dim, rerounded=alt, **kw))
            continue
        if (
            before is None
            or type_error(new) is not None
            or not (before.shape == ref.shape == new.shape)
            or not (before.dtype == ref.dtype == new.dtype)
        ):
            results.append(compare_tensors(name, ref, new, rerounded=alt, **kw))
            continue
        before, ref = before.to(new.device), ref.to(new.device)
        changed = (ref != before) | (new != before)
        count = int(changed.sum())
        if count == 0:
            results.append({"name": name, "ok": True, "changed_elements": 0, "max_abs_err": 0.0})
            continue
        alt = _like(alt, ref)
        alt = None if alt is None else alt.to(new.device)[changed]
        result = compare_tensors(name, ref[changed], new[changed], rerounded=alt, **kw)
        result["changed_elements"] = count
        results.append(result)
    return results
