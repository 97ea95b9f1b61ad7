"""The scale-rule guard of block-scaled activations, the drop-in for the evaluator's
``kernel_agent.kernels.scale_guard`` (src/kernel_agent/kernels/scale_guard.py).

A candidate of ``fp8_mx`` or ``fp4_w4a4`` precision exposes its activation quantiser as a
module-level ``quantize_activations(x)``. The guard feeds it two inputs of the same shape, the
captured activation of the busiest case and a stress input whose block maxima sit where a
saturating scale rule shows, and rejects the candidate when its scales saturate (W4A4: or
flush non-zero blocks to scale 0) or the call fails. Every check is a GPU reduction of this
library: the scale-rule checks (``kab_mxfp8_saturation``, ``kab_fp4_scale_check``) and the
outlier statistics of the captured input (``kab_outlier_stats``).

What is kept from the reference, because the evaluator and ``integrity.Snapshot`` read it:
the names ``QUANTIZER`` / ``GUARDED`` and their values, the notes of an unchecked candidate,
the report's keys and the error texts (scale_guard.py:64-82, 139-188).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any, Callable, Iterator

import torch

from .. import _native as nat
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


# ------------------------------------------------------------------ the two scale rules


def _inspect_mxfp8(sample: torch.Tensor, out: Any, fmt: str | None) -> tuple[dict[str, Any], str | None]:
    """``(codes, scales)``: the MXFP8 saturation summary and the problem, if any."""
    scales = out[1]
    found = quant.mxfp8_saturation(sample, scales)
    return _pick(found, _MXFP8_KEYS), quant.mxfp8_scale_problem(sample, scales)


def _inspect_fp4(sample: torch.Tensor, out: Any, fmt: str | None) -> tuple[dict[str, Any], str | None]:
    """``(codes, scales[, outer[, quantised]])``: the W4A4 scale check of the activations the
    quantiser actually quantised (its fourth result when it rotates its input first)."""
    scales = out[1]
    outer = out[2] if len(out) > 2 else None
    quantised = out[3] if len(out) > 3 and out[3] is not None else sample
    if quantised.shape[-1] != sample.shape[-1] or quantised.numel() != sample.numel():
        raise ValueError(f"the quantised activations {tuple(quantised.shape)} are not of the input's size")
    found = quant.fp4_scale_check(quantised, scales, outer, fmt)
    return _pick(found, _FP4_KEYS), quant.fp4_scale_problem(quantised, scales, outer, fmt)


_MXFP8_KEYS = ("blocks", "saturated", "worst_ratio", "coarser")
_FP4_KEYS = ("format", "blocks", "saturated", "worst_ratio", "underflow", "coarser")


def _pick(found: dict[str, Any], keys: tuple[str, ...]) -> dict[str, Any]:
    return {key: found[key] for key in keys}


@dataclass(frozen=True)
class _Precision:
    """How the guard treats one precision: the stress input of a shape, how a quantiser's
    output is judged, and whether the stress input depends on the captured run's format."""

    stress: Callable[[tuple[int, ...], str, torch.dtype, torch.device], torch.Tensor]
    inspect: Callable[[torch.Tensor, Any, str | None], tuple[dict[str, Any], str | None]]
    formatted: bool


_PRECISIONS = {
    "fp8_mx": _Precision(
        stress=lambda shape, fmt, dtype, device: quant.mxfp8_stress_input(shape, dtype=dtype, device=device),
        inspect=_inspect_mxfp8,
        formatted=False,
    ),
    "fp4_w4a4": _Precision(
        stress=lambda shape, fmt, dtype, device: quant.fp4_stress_input(shape, fmt, dtype=dtype, device=device),
        inspect=_inspect_fp4,
        formatted=True,
    ),
}


# ------------------------------------------------------------------ inputs


def _quantisable(value: Any, block: int) -> bool:
    return (isinstance(value, torch.Tensor) and value.is_floating_point() and value.dim() >= 2
            and value.numel() > 0 and value.shape[-1] % block == 0)


def _arguments(case: dict[str, Any]) -> Iterator[Any]:
    yield from case.get("args", ())
    yield from (case.get("kwargs") or {}).values()


def activation(cases: list[dict[str, Any]], block: int = quant.MX_BLOCK) -> torch.Tensor | None:
    """scale_guard.py:85-100: the first floating-point tensor argument (at least 2-D, last
    dimension a multiple of ``block``, not empty) of the case called most often (the first
    such case on a tie), or None."""
    busiest_first = sorted(cases, key=lambda case: int(case.get("count") or 0), reverse=True)
    # sorted(reverse=True) keeps the input order of equal counts, as the reference's ranking does
    return next((v for case in busiest_first for v in _arguments(case) if _quantisable(v, block)), None)


def outliers(x: torch.Tensor) -> dict[str, float]:
    """scale_guard.py:103-118: ``crest``, the largest ``amax / RMS`` of a row with a non-zero
    RMS, and ``channel_ratio``, the largest channel amax over the median channel's, of
    ``x [..., K]`` (non-finite values count as 0). One GPU pass (``kab_outlier_stats``) gives
    the rows' sums of squares and maxima and the channels' maxima; the ratios are taken from
    those few numbers."""
    nat.require_cuda(x)
    k = x.shape[-1]
    rows = quant._rows(x.detach())
    if rows.dtype not in nat.DTYPES:
        rows = rows.float()
    if rows.stride(-1) != 1 or rows.stride(0) % 8 or rows.data_ptr() % 16 or k % 8:
        rows = rows.contiguous()
        if k % 8:  # the kernel reads 8 elements at a time: zero columns change no statistic
            rows = torch.nn.functional.pad(rows, (0, 8 - k % 8))
    n, width = rows.shape
    sumsq = torch.empty(n, dtype=torch.float64, device=x.device)
    row_max = torch.empty(n, dtype=torch.float32, device=x.device)
    col_max = torch.empty(width, dtype=torch.float32, device=x.device)
    nat.call("kab_outlier_stats", rows.data_ptr(), nat.dtype_code(rows), n, width, rows.stride(0),
             sumsq.data_ptr(), row_max.data_ptr(), col_max.data_ptr(), nat.stream_of(rows))
    rms = (sumsq / k).sqrt().float()
    live = rms > 0
    crest = (row_max / rms.clamp_min(1e-30))[live]
    channels = col_max[:k]
    median = float(channels.median())
    return {
        "crest": round(float(crest.max()), 1) if crest.numel() else 0.0,
        "channel_ratio": round(float(channels.max()) / median, 1) if median > 0 else 0.0,
    }


# ------------------------------------------------------------------ the guard


def _run(fn: Callable[[torch.Tensor], Any], label: str, sample: torch.Tensor, rule: _Precision,
         fmt: str | None, precision: str) -> tuple[str | None, dict[str, Any] | None, str | None]:
    """One input through the candidate's quantiser: (its format, its summary, the error text
    or None). Any exception of the candidate's function or of the check is the error."""
    what = f"{QUANTIZER} on the {label} input {list(sample.shape)} {sample.dtype}"
    try:
        with torch.inference_mode():
            out = fn(sample.clone())
        if rule.formatted:
            fmt = fmt or quant.fp4_format_of(sample.shape[-1], out[1])
        summary, problem = rule.inspect(sample, out, fmt)
    except Exception as exc:  # the candidate's function, or scales of the wrong shape
        return fmt, None, f"{what}: {type(exc).__name__}: {exc}"[:600]
    return fmt, summary, None if problem is None else f"{what}: {problem}"


def check(module: Any, cases: list[dict[str, Any]], precision: str = "fp8_mx") -> dict[str, Any]:
    """scale_guard.py:139-188: the scale-rule report of a candidate: ``ok``, ``checked``, per
    input (``captured``, then ``stress``) its summary, ``outliers`` of the captured input, and
    ``error`` with the ``input`` it came from when the candidate fails; ``note`` when the rule
    went unchecked."""
    block = GUARDED.get(precision, quant.MX_BLOCK)
    rule = _PRECISIONS.get(precision, _PRECISIONS["fp8_mx"])
    captured = activation(cases, block)
    report: dict[str, Any] = {"ok": True, "checked": False}
    if captured is not None:
        report["outliers"] = outliers(captured)
    fn = getattr(module, QUANTIZER, None)
    if not callable(fn):
        report["note"] = f"no module-level {QUANTIZER}(x) -> {_RULES.get(precision, _RULES['fp8_mx'])} in the candidate"
        return report
    if captured is None:
        report["note"] = f"no floating-point input with K a multiple of {block}: nothing to quantise"
        return report
    report["checked"] = True
    fmt: str | None = None  # W4A4: the captured run's format decides the stress input's
    shape = tuple(captured.shape)
    for label in ("captured", "stress"):
        sample = captured if label == "captured" else rule.stress(shape, fmt or "nvfp4", captured.dtype, captured.device)
        fmt, summary, error = _run(fn, label, sample, rule, fmt, precision)
        if summary is not None:
            report[label] = summary
        if error is not None:
            report.update(ok=False, input=label, error=error)
            return report
    return report
