"""The scale-rule guard of block-scaled activations (src/kernel_agent/kernels/scale_guard.py),
on the GPU checks of :mod:`kernel_agent_b200.kernels.quant`.

A candidate of ``fp8_mx`` or ``fp4_w4a4`` precision exposes its activation quantiser as a
module-level ``quantize_activations(x)``; :func:`check` runs it on the captured input of the
main case and on a stress input of the same shape and rejects the candidate when its scales
saturate (or, W4A4, flush non-zero blocks to scale 0) or the quantiser fails, with the same
report as the reference (scale_guard.py:139-188). The MXFP8 / FP4 checks are one GPU
reduction each (``kab_mxfp8_saturation``, ``kab_fp4_scale_check``).
"""

from __future__ import annotations

from typing import Any

import torch

from . import quant

#: The module-level function of a candidate the guard runs (scale_guard.py:64).
QUANTIZER = "quantize_activations"
#: The precisions whose candidates the guard checks, and the block of K their activation
#: input must be a whole number of (scale_guard.py:67).
GUARDED = {"fp8_mx": quant.MX_BLOCK, "fp4_w4a4": quant.FP4_FORMATS["nvfp4"][0]}
_RULES = {
    "fp8_mx": (
        "(codes, scales): its MXFP8 scale rule is not checked (it must be "
        "2^ceil(log2(amax / 448)); the OCP rule 2^(floor(log2 amax) - 8) saturates block "
        "maxima above 448 x scale)"
    ),
    "fp4_w4a4": (
        "(codes, scales, outer): its W4A4 scale rule is not checked (NVFP4: the e4m3 block "
        "scale bmax / (outer x 6) rounded to nearest, outer = amax / (6 x 448); MXFP4: "
        "2^ceil(log2(amax / 6)))"
    ),
}


def activation(cases: list[dict[str, Any]], block: int = quant.MX_BLOCK) -> torch.Tensor | None:
    """scale_guard.py:85-100: the first floating-point tensor argument (at least 2-D, last
    dimension a multiple of ``block``, not empty) of the case with the most calls, or None."""
    for case in sorted(cases, key=lambda c: -int(c.get("count") or 0)):
        for value in [*case.get("args", ()), *(case.get("kwargs") or {}).values()]:
            if (isinstance(value, torch.Tensor) and value.is_floating_point() and value.dim() >= 2
                    and value.shape[-1] % block == 0 and value.numel() > 0):
                return value
    return None


def outliers(x: torch.Tensor) -> dict[str, float]:
    """scale_guard.py:103-118: ``crest`` (the largest row amax / RMS) and ``channel_ratio``
    (the largest channel amax over the median channel's) of ``x [..., K]``."""
    a = x.detach().reshape(-1, x.shape[-1]).float()
    a = torch.where(torch.isfinite(a), a, torch.zeros_like(a))
    rms = a.pow(2).mean(dim=1).sqrt()
    crest = a.abs().amax(dim=1) / rms.clamp_min(1e-30)
    channel = a.abs().amax(dim=0)
    median = float(channel.median())
    live = rms > 0
    return {
        "crest": round(float(crest[live].max()), 1) if bool(live.any()) else 0.0,
        "channel_ratio": round(float(channel.max()) / median, 1) if median > 0 else 0.0,
    }


def _mxfp8(sample: torch.Tensor, out: Any) -> tuple[dict[str, Any], str | None]:
    scales = out[1]
    found = quant.mxfp8_saturation(sample, scales)
    summary = {k: found[k] for k in ("blocks", "saturated", "worst_ratio", "coarser")}
    return summary, quant.mxfp8_scale_problem(sample, scales)


def _fp4(sample: torch.Tensor, out: Any, fmt: str | None) -> tuple[dict[str, Any], str | None]:
    scales, outer = out[1], (out[2] if len(out) > 2 else None)
    x = out[3] if len(out) > 3 and out[3] is not None else sample
    if tuple(x.shape[-1:]) != tuple(sample.shape[-1:]) or x.numel() != sample.numel():
        raise ValueError(f"the quantised activations {tuple(x.shape)} are not of the input's size")
    found = quant.fp4_scale_check(x, scales, outer, fmt)
    keys = ("format", "blocks", "saturated", "worst_ratio", "underflow", "coarser")
    return {k: found[k] for k in keys}, quant.fp4_scale_problem(x, scales, outer, fmt)


def check(module: Any, cases: list[dict[str, Any]], precision: str = "fp8_mx") -> dict[str, Any]:
    """scale_guard.py:139-188: the scale-rule report of a candidate: ``ok``, ``checked``, per
    input (``captured``, ``stress``) its summary, ``outliers`` of the captured input, and
    ``error`` (with ``input``) when it fails; ``note`` when the rule went unchecked."""
    block = GUARDED.get(precision, quant.MX_BLOCK)
    x = activation(cases, block)
    report: dict[str, Any] = {"ok": True, "checked": False}
    if x is not None:
        report["outliers"] = outliers(x)
    fn = getattr(module, QUANTIZER, None)
    if not callable(fn):
        rule = _RULES.get(precision, _RULES["fp8_mx"])
        report["note"] = f"no module-level {QUANTIZER}(x) -> {rule} in the candidate"
        return report
    if x is None:
        report["note"] = f"no floating-point input with K a multiple of {block}: nothing to quantise"
        return report
    report["checked"] = True
    fmt: str | None = None
    for name in ("captured", "stress"):
        if name == "captured":
            sample = x
        elif precision == "fp4_w4a4":
            sample = quant.fp4_stress_input(tuple(x.shape), fmt or "nvfp4", dtype=x.dtype, device=x.device)
        else:
            sample = quant.mxfp8_stress_input(tuple(x.shape), dtype=x.dtype, device=x.device)
        what = f"{QUANTIZER} on the {name} input {list(sample.shape)} {sample.dtype}"
        try:
            with torch.inference_mode():
                out = fn(sample.clone())
            if precision == "fp4_w4a4":
                fmt = fmt or quant.fp4_format_of(sample.shape[-1], out[1])
                summary, problem = _fp4(sample, out, fmt)
            else:
                summary, problem = _mxfp8(sample, out)
        except Exception as exc:  # the candidate's function, or scales of the wrong shape
            report.update(ok=False, input=name, error=f"{what}: {type(exc).__name__}: {exc}"[:600])
            return report
        report[name] = summary
        if problem is not None:
            report.update(ok=False, input=name, error=f"{what}: {problem}")
            return report
    return report
