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
    """compare.py:793-803: ``rerounded`` (detached) if it is a plain tensor of ``ref``'s shape
    and dtype, else None."""
    usable = (isinstance(rerounded, torch.Tensor) and type_error(rerounded) is None
              and rerounded.shape == ref.shape and rerounded.dtype == ref.dtype)
    return rerounded.detach() if usable else None


# ------------------------------------------------------------------ caches and structures
#
# compare.py:806-1182. A tier judges part of an output when the call changed part of an
# input: a cache grown along one dimension (the appended rows), rows written into an input
# of the same shape (the box they span), or an argument updated in place (the elements either
# side changed). The rest must be as the reference left it. Which elements differ from the
# call's input is one GPU pass each (``kab_diff_census``: a count and, when asked, a mask of
# the differing elements and, per dimension, the indices that hold one); the kept parts go
# through :func:`compare_tensors`.


@dataclasses.dataclass
class _Census:
    """The elements of a region that differ from the base tensor: how many, and (when asked)
    a boolean mask of the region and per-dimension index flags."""

    count: int
    mask: torch.Tensor | None = None
    hits: list[torch.Tensor] | None = None


def _census_dtype(t: torch.Tensor) -> tuple[torch.Tensor, int]:
    """The tensor as the census reads it and its type code: floats by value, integers and
    booleans by their bits."""
    if t.dtype in nat.DTYPES:
        return t, nat.DTYPES[t.dtype]
    if t.dtype == torch.float64:
        return t, nat.KAB_DIFF_F64
    if t.is_floating_point():
        return t.float(), nat.KAB_F32  # 1-byte floats: their fp32 values are exact
    if t.element_size() not in nat.KAB_DIFF_BITS:
        raise ValueError(f"the difference census does not read {t.dtype} tensors")
    return t, nat.KAB_DIFF_BITS[t.element_size()]


def _census(a: torch.Tensor, base: torch.Tensor, *, also: torch.Tensor | None = None, nan_equal: bool = True,
            dim: int = 0, length: int | None = None, a_off: int = 0, base_off: int = 0, mask: bool = False,
            hits: bool = False, outside: list[torch.Tensor] | None = None) -> _Census:
    """Which elements of ``a`` (or of ``a`` or ``also``, laid out like ``a``) differ from
    ``base`` over ``length`` indices along ``dim`` (from ``a_off`` in ``a``, ``base_off`` in
    ``base``; the whole dimension by default). ``nan_equal``: NaN equals NaN; else IEEE
    ``!=``. ``outside``: per dimension the flags of a box whose elements are not counted."""
    dev = nat.require_cuda(a)
    shape0 = tuple(a.shape)
    a, code = _census_dtype(a.detach().contiguous())
    base = _census_dtype(base.detach().to(dev).contiguous())[0]
    if also is not None:
        also = _census_dtype(also.detach().to(dev).contiguous())[0]
    shape = list(a.shape) or [1]
    dim = dim % len(shape)
    length = shape[dim] if length is None else length
    region = shape[:dim] + [length] + shape[dim + 1:]
    p = nat.KabDiffParams()
    p.a, p.b, p.base = a.data_ptr(), nat.ptr(also), base.data_ptr()
    p.dtype, p.nan_equal = code, int(nan_equal)
    p.outer, p.len, p.inner = math.prod(shape[:dim]), length, math.prod(shape[dim + 1:])
    p.a_dim, p.a_off = shape[dim], a_off
    p.base_dim, p.base_off = (list(base.shape) or [1])[dim], base_off
    flags = box = None
    if hits or outside is not None:
        if len(region) > nat.KAB_DIFF_MAXDIM:
            raise ValueError(f"a census over {len(region)} dimensions (at most {nat.KAB_DIFF_MAXDIM})")
        p.ndim = len(region)
        for k, n in enumerate(region):
            p.shape[k] = n
        if hits:
            flags = torch.zeros(sum(region), dtype=torch.uint8, device=dev)
            p.hits = flags.data_ptr()
        if outside is not None:
            box = torch.cat([f.to(dev, torch.uint8).reshape(-1) for f in outside])
            p.box = box.data_ptr()
    marks = torch.empty(region, dtype=torch.uint8, device=dev) if mask else None
    p.mask = nat.ptr(marks)
    count = torch.empty(1, dtype=torch.int64, device=dev)
    nat.call("kab_diff_census", ctypes.byref(p), count.data_ptr(), nat.stream_of(a))
    found = _Census(int(count.item()))  # one device-to-host read
    if marks is not None:
        found.mask = marks.bool().reshape(shape0[:dim] + (length,) + shape0[dim + 1:]) if shape0 else marks.bool().reshape(())
    if flags is not None:
        found.hits = [f.bool() for f in flags.split(region)]
    return found


def _mismatched(new: Any, ref: torch.Tensor) -> bool:
    """compare.py:860-867 / 980-987: a candidate compared whole (its error) rather than by part."""
    return (type_error(new) is not None or new.shape != ref.shape or new.dtype != ref.dtype
            or new.layout != ref.layout or new.device.type != ref.device.type)


def _settle(result: dict[str, Any], problems: list[str]) -> dict[str, Any]:
    """The verdict of a comparison by parts: its problems, or ok."""
    result.pop("error", None)
    if problems:
        result["error"] = "; ".join(problems)
    result["ok"] = not problems
    return result


def _channels_floor(ref: torch.Tensor, perturbed: bool) -> torch.Tensor | None:
    """compare.py:582-589 on the whole reference, as a per-channel floor ``[C]`` for the part
    a tier judges (on redrawn inputs only)."""
    return _channel_rms_of(ref.float().contiguous()) if perturbed else None


def grown_dim(before: Any, after: Any) -> int | None:
    """compare.py:806-825: the one dimension along which ``after`` is ``before`` grown (both
    floating-point, strided, one dtype and rank, ``before`` not empty), or None."""
    if not isinstance(before, torch.Tensor) or not isinstance(after, torch.Tensor):
        return None
    comparable = (before.is_floating_point() and before.dtype == after.dtype and before.dim() == after.dim()
                  and before.layout == torch.strided == after.layout and before.numel() > 0)
    if not comparable:
        return None
    grew = [d for d, (b, a) in enumerate(zip(before.shape, after.shape)) if b != a]
    return grew[0] if len(grew) == 1 and after.shape[grew[0]] > before.shape[grew[0]] else None


def compare_grown(name, before, ref, new, dim, *, tier=None, perturbed=False, input_scale=1.0,
                  rerounded=None) -> dict[str, Any]:
    """compare.py:833-915: ``new`` against ``ref``, both ``before`` grown along ``dim``: the
    appended rows on their own with the tier's checks, and the kept part: bit for bit where
    the reference kept it, else the elements either side changed."""
    options = {"tier": tier, "perturbed": perturbed, "input_scale": input_scale}
    if _mismatched(new, ref):
        return compare_tensors(name, ref, new, rerounded=rerounded, **options)
    dev = new.device
    spread = _like(rerounded, ref)
    ref, before, new = ref.detach().to(dev), before.detach().to(dev), new.detach()
    old = before.shape[dim]
    grown = ref.shape[dim] - old

    def appended(t: torch.Tensor) -> torch.Tensor:
        return t.narrow(dim, old, grown)

    floor = _channels_floor(ref, perturbed)
    if floor is not None and dim == ref.dim() - 1:  # grown along the channels themselves
        floor = floor.narrow(0, old, grown)
    result = compare_tensors(name, appended(ref), appended(new), channel_rms=floor,
                             rerounded=None if spread is None else appended(spread.to(dev)), **options)
    result["grown"] = {"dim": dim, "kept": old, "appended": grown}
    problems = []
    if "error" in result:
        plural = "s" if grown != 1 else ""
        problems.append(f"the {grown} appended row{plural} along dim {dim} (after {old} kept): {result['error']}")
    # the kept part: did the reference leave it as the input?
    if _census(ref, before, dim=dim, length=old).count == 0:
        drift = _census(new, before, dim=dim, length=old).count
        result["kept_changed"] = drift
        if drift:
            problems.append(f"{drift} of the {before.numel()} elements of the {old} kept rows along dim {dim} "
                            "changed; the reference keeps them as they were (it only appends)")
    else:
        either = _census(ref, before, also=new, dim=dim, length=old, mask=True)
        pick = either.mask

        def kept(t: torch.Tensor) -> torch.Tensor:
            return t.narrow(dim, 0, old)[pick]

        judged = compare_tensors(name, kept(ref), kept(new),
                                 rerounded=None if spread is None else kept(spread.to(dev)), **options)
        result["changed_elements"] = either.count
        if not judged["ok"]:
            problems.append(f"the {either.count} changed elements of the {old} kept rows: {judged['error']}")
    return _settle(result, problems)


def written_box(before: Any, after: Any) -> list[torch.Tensor] | None:
    """compare.py:918-953: per dimension, the indices of the box of rows a call wrote into
    ``before`` to give ``after`` (same shape, floating-point, strided, not empty); None when
    nothing differs, or the differences do not fill WRITTEN_MIN_DENSITY of a box that spans a
    whole dimension of more than one element and at most WRITTEN_MAX_FRACTION of the tensor."""
    if not isinstance(before, torch.Tensor) or not isinstance(after, torch.Tensor):
        return None
    comparable = (before.is_floating_point() and before.dtype == after.dtype and before.shape == after.shape
                  and before.layout == torch.strided == after.layout and before.dim() > 0 and before.numel() > 0)
    if not comparable or before.dim() > nat.KAB_DIFF_MAXDIM:  # more dimensions than the census takes:
        return None                                                # compared whole
    found = _census(after, before.to(after.device), hits=True)
    if found.count == 0:  # the input itself: compared whole
        return None
    extent = [int(h.sum()) for h in found.hits]
    spans_a_row = any(e == n > 1 for e, n in zip(extent, after.shape))
    area = math.prod(extent)
    if area > WRITTEN_MAX_FRACTION * after.numel() or found.count < WRITTEN_MIN_DENSITY * area or not spans_a_row:
        return None
    return [h.nonzero().flatten() for h in found.hits]


def compare_written(name, before, ref, new, box, *, tier=None, perturbed=False, input_scale=1.0,
                    rerounded=None) -> dict[str, Any]:
    """compare.py:956-1034: rows written into an input: the box (``box``: its indices per
    dimension) with the tier's checks, every element outside it bit for bit as before."""
    options = {"tier": tier, "perturbed": perturbed, "input_scale": input_scale}
    if _mismatched(new, ref):
        return compare_tensors(name, ref, new, rerounded=rerounded, **options)
    dev = new.device
    spread = _like(rerounded, ref)
    ref, before, new = ref.detach().to(dev), before.detach().to(dev), new.detach()
    box = [index.to(dev) for index in box]

    def inside(t: torch.Tensor) -> torch.Tensor:
        for d, index in enumerate(box):
            if index.numel() < t.shape[d]:
                t = t.index_select(d, index)
        return t

    floor = _channels_floor(ref, perturbed)
    if floor is not None and box[-1].numel() < ref.shape[-1]:  # written along the channels
        floor = floor.index_select(0, box[-1])
    result = compare_tensors(name, inside(ref), inside(new), channel_rms=floor,
                             rerounded=None if spread is None else inside(spread.to(dev)), **options)
    extent = [int(index.numel()) for index in box]
    written = f"written {extent} of {list(ref.shape)}"
    result["written"] = {"box": extent, "of": list(ref.shape)}
    problems = []
    if "error" in result:
        problems.append(f"the {written} (where the reference changed the input): {result['error']}")
    member = []
    for d, index in enumerate(box):
        flag = torch.zeros(ref.shape[d], dtype=torch.bool, device=dev)
        flag[index] = True
        member.append(flag)
    drift = _census(new, before, outside=member).count
    result["kept_changed"] = drift
    if drift:
        problems.append(f"{drift} of the {ref.numel() - math.prod(extent)} elements outside the {written} "
                        "changed; the reference keeps them as they were (it only writes the box)")
    return _settle(result, problems)


def _grows_from(before: torch.Tensor, ref: torch.Tensor) -> int | None:
    """The dimension along which ``ref`` grows ``before`` with its leading part there equal to
    ``before`` (NaN as NaN), or None."""
    dim = grown_dim(before, ref)
    if dim is None:
        return None
    return dim if _census(ref, before, dim=dim, length=before.shape[dim]).count == 0 else None


def compare_output(name, ref, new, inputs=(), *, tier=None, perturbed=False, input_scale=1.0,
                   rerounded=None) -> dict[str, Any]:
    """compare.py:1037-1071: an output that grows one of the call's inputs
    (:func:`compare_grown`), one with rows written into one of them (:func:`compare_written`),
    else the whole tensor (:func:`compare_tensors`)."""
    options = {"tier": tier, "perturbed": perturbed, "input_scale": input_scale, "rerounded": rerounded}
    grown = next(((src, dim) for src in inputs if (dim := _grows_from(src, ref)) is not None), None)
    if grown is not None:
        return compare_grown(name, grown[0], ref, new, grown[1], **options)
    written = next(((src, box) for src in inputs if (box := written_box(src, ref)) is not None), None)
    if written is not None:
        return compare_written(name, written[0], ref, new, written[1], **options)
    return compare_tensors(name, ref, new, **options)


def compare_structures(ref, new, prefix: str = "out", *, inputs=None, tier=None, perturbed=False,
                       input_scale=1.0, rerounded=None) -> list[dict[str, Any]]:
    """compare.py:1074-1103: the candidate's output against the reference's, tensor by
    tensor (names from :func:`flatten`), each through :func:`compare_output`."""
    candidate = flatten(new, prefix)
    redrawn = flatten(rerounded, prefix)
    sources = list(flatten(inputs, "in").values())
    options = {"tier": tier, "perturbed": perturbed, "input_scale": input_scale}

    def one(name: str, tensor: torch.Tensor) -> dict[str, Any]:
        if name not in candidate:
            return {"name": name, "ok": False, "error": "missing in candidate output"}
        return compare_output(name, tensor, candidate[name], sources, rerounded=redrawn.get(name), **options)

    return [one(name, tensor) for name, tensor in flatten(ref, prefix).items()]


def compare_side_effects(pre, ref_post, new_post, prefix: str = "args", *, tier=None,
                         perturbed=False, input_scale=1.0, rerounded=None) -> list[dict[str, Any]]:
    """compare.py:1106-1137: the post-call state of a call's arguments."""
    return compare_side_effects_flat(
        flatten(pre, prefix), flatten(ref_post, prefix), flatten(new_post, prefix), tier=tier,
        perturbed=perturbed, input_scale=input_scale, rerounded_flat=flatten(rerounded, prefix),
    )


def _updated_in_place(before: Any, ref: torch.Tensor, new: Any) -> bool:
    """Whether an argument kept its shape and dtype on both sides (an in-place update)."""
    return (before is not None and type_error(new) is None and before.shape == ref.shape == new.shape
            and before.dtype == ref.dtype == new.dtype)


def compare_side_effects_flat(pre_flat, ref_flat, new_flat, *, tier=None, perturbed=False,
                              input_scale=1.0, rerounded_flat=None) -> list[dict[str, Any]]:
    """compare.py:1140-1182: each argument the reference's call left: grown (by
    :func:`compare_grown`), updated in place (the elements either side changed, by IEEE
    ``!=``, judged alone), or compared whole."""
    options = {"tier": tier, "perturbed": perturbed, "input_scale": input_scale}
    redrawn = rerounded_flat or {}

    def one(name: str, ref: torch.Tensor) -> dict[str, Any]:
        new = new_flat.get(name)
        if new is None:
            return {"name": name, "ok": False, "error": "missing in candidate arguments"}
        spread = redrawn.get(name)
        before = pre_flat.get(name)
        dim = grown_dim(before, ref) if before is not None else None
        if dim is not None:
            return compare_grown(name, before, ref, new, dim, rerounded=spread, **options)
        if not _updated_in_place(before, ref, new):
            return compare_tensors(name, ref, new, rerounded=spread, **options)
        dev = new.device
        ref_d, before_d = ref.to(dev), before.to(dev)
        either = _census(ref_d, before_d, also=new, nan_equal=False, mask=True)
        if either.count == 0:
            return {"name": name, "ok": True, "changed_elements": 0, "max_abs_err": 0.0}
        alt = _like(spread, ref)
        pick = either.mask
        result = compare_tensors(name, ref_d[pick], new[pick],
                                 rerounded=None if alt is None else alt.to(dev)[pick], **options)
        result["changed_elements"] = either.count
        return result

    return [one(name, ref) for name, ref in ref_flat.items()]
