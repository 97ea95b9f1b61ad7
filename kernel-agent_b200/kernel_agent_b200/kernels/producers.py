"""Fused quantise producers, the GPU counterparts of kernel-agent's example producers
(``src/kernel_agent/agent/examples/triton_fp8_producers.py:177-222`` and
``triton_fp4_producers.py:369-434``): ``silu(gate) * up`` (or a plain row) quantised in the
producer's epilogue, so the next GEMM reads one byte (FP8) or half a byte (FP4) per
activation and no bf16 intermediate is written; and RMSNorm producers
(``triton_fp8_producers.py:191-202``, ``triton_fp4_producers.py:384-405``).

The values quantised are eager's (``F.silu`` rounded to the input dtype, the product
rounded again); codes and scales equal ``quant.quantize_*`` of those values bit for bit.
``out`` (optional, ``[rows, K]`` in the input dtype) also receives the producer's own output.
``unbiased`` (FP4): also the epilogue's per-token scale ``outer * quant.fp4_bias_correction``
of that output (a fourth result), as the reference's producers return it.

The RMSNorm producers (``r = rsqrt(sum(x^2) / K + eps)`` in fp32, ``h = dtype(dtype(x * r) *
weight)``) norm and quantise each row in one pass over ``x`` (``kab_rmsnorm_quant_fp8``,
``kab_rmsnorm_quant_fp4``), ``h`` kept in registers and written only to ``out``; FP8 rows
wider than 16384 and fp32 FP4 rows take two passes (``kab_rmsnorm`` into ``out`` or a
temporary, then the quantisers). Either way the codes are
exactly those of ``h``, and ``h`` is eager's RMSNorm up to the order of the sum of squares
and the last bit of ``rsqrt``.
"""

from __future__ import annotations

import torch

from .. import _native as nat
from . import quant as q

_E4M3 = torch.float8_e4m3fn


def _split(gate: torch.Tensor, up: torch.Tensor | None) -> tuple[torch.Tensor, torch.Tensor]:
    """(gate, up) rows; without ``up``, ``gate`` is the merged ``[..., 2F]`` gate|up output."""
    g2 = q._rows(gate)
    if up is None:
        f = g2.shape[1] // 2
        return g2[:, :f], g2[:, f:]
    u2 = q._rows(up)
    if u2.shape != g2.shape:
        raise ValueError(f"gate {tuple(g2.shape)} and up {tuple(u2.shape)} differ")
    return g2, u2


def _check_out(out: torch.Tensor | None, like: torch.Tensor) -> None:
    if out is not None and (out.shape != like.shape or out.dtype != like.dtype or not out.is_contiguous()):
        raise ValueError(f"out must be a contiguous {like.dtype} tensor of shape {tuple(like.shape)}")


def quantize_rows(x: torch.Tensor, mx: bool = False, blocked: bool = False):
    """``(codes, scales)`` of ``x [..., K]`` (triton_fp8_producers.py:177-188): per token
    (e4m3 + fp32 ``[rows]``) or MXFP8 with ``mx`` (e8m0 bytes ``[rows, K / 32]``, or the
    swizzled 128 x 4 layout with ``blocked``)."""
    nat.require_cuda(x)
    x2 = q._rows(q._input(x))
    if mx:
        return q._mxfp8(x2, "ceil", swizzle=blocked)
    return q._fp8_rows(x2)


def silu_mul_fp8(gate: torch.Tensor, up: torch.Tensor | None = None, mx: bool = False,
                 blocked: bool = False, out: torch.Tensor | None = None):
    """``(codes, scales)`` of ``F.silu(gate) * up`` (bf16 / fp16), quantised in the epilogue
    (triton_fp8_producers.py:205-221)."""
    nat.require_cuda(gate, up)
    g2, u2 = _split(gate, up)
    if g2.dtype not in (torch.bfloat16, torch.float16):
        raise ValueError("the fused SiLU * up producer takes bf16 or fp16")
    _check_out(out, g2.new_empty(g2.shape) if out is not None else g2)
    if mx:
        if g2.shape[1] % q.MX_BLOCK:
            raise ValueError(f"the last dimension {g2.shape[1]} is not a multiple of the MXFP8 block (32)")
        return q._mxfp8(g2, "ceil", up=u2, swizzle=blocked, h=out)
    return q._fp8_rows(g2, up=u2, h=out)


def _fp4_block(k: int, mx: bool) -> str:
    fmt = "mxfp4" if mx else "nvfp4"
    block = q.FP4_FORMATS[fmt][0]
    if k % block:
        raise ValueError(f"the last dimension {k} is not a multiple of the {fmt} block ({block})")
    return fmt


def _result_fp4(h2: torch.Tensor, res, fmt: str, swizzle: bool, unbiased: bool):
    """(codes, scales, outer) or, with ``unbiased``, (codes, scales, outer, outer * c) where c
    is ``quant.fp4_bias_correction`` of h2 (triton_fp4_producers.py:364-366)."""
    if not unbiased:
        return res
    codes, scales, outer = res
    c = q._bias_correction(h2, codes, scales, fmt, outer, swizzled=swizzle)
    return codes, scales, outer, outer * c


def quantize_rows_fp4(x: torch.Tensor, mx: bool = False, swizzle: bool = False, unbiased: bool = False):
    """``(codes, scales, outer)`` of ``x [..., K]`` (triton_fp4_producers.py:369-381): NVFP4
    (per-token outer scale) or MXFP4 with ``mx``; scales row-major or swizzled; ``unbiased``:
    and the epilogue's per-token scale (fourth)."""
    nat.require_cuda(x)
    fmt = _fp4_block(x.shape[-1], mx)
    x2 = q._rows(q._input(x))
    return _result_fp4(x2, q._fp4(x2, fmt, nat.KAB_FP4_TOKEN, swizzle=swizzle), fmt, swizzle, unbiased)


def silu_mul_fp4(gate: torch.Tensor, up: torch.Tensor | None = None, mx: bool = False,
                 swizzle: bool = False, out: torch.Tensor | None = None, unbiased: bool = False):
    """``(codes, scales, outer)`` of ``F.silu(gate) * up`` quantised to NVFP4 (MXFP4 with
    ``mx``) in the epilogue (triton_fp4_producers.py:408-434); ``unbiased``: and the
    epilogue's per-token scale (fourth; the product is then also written, to ``out`` or a
    temporary)."""
    nat.require_cuda(gate, up)
    g2, u2 = _split(gate, up)
    if g2.dtype not in (torch.bfloat16, torch.float16):
        raise ValueError("the fused SiLU * up producer takes bf16 or fp16")
    fmt = _fp4_block(g2.shape[1], mx)
    _check_out(out, g2)
    h = out if out is not None or not unbiased else torch.empty(g2.shape, dtype=g2.dtype, device=g2.device)
    res = q._fp4(g2, fmt, nat.KAB_FP4_TOKEN, up=u2, swizzle=swizzle, h=h)
    return _result_fp4(h, res, fmt, swizzle, unbiased) if unbiased else res


def _rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float, out: torch.Tensor | None) -> torch.Tensor:
    """h = RMSNorm(x) * weight in x's dtype, [rows, K], into ``out`` or a new tensor."""
    nat.require_cuda(x, weight)
    x2 = q._rows(q._input(x))
    m, k = x2.shape
    if k % 8:
        raise ValueError(f"the last dimension {k} is not a multiple of 8")
    w = weight.to(device=x2.device, dtype=x2.dtype).reshape(-1).contiguous()
    if w.numel() != k:
        raise ValueError(f"weight has {w.numel()} elements, expected {k}")
    _check_out(out, x2)
    h = torch.empty(m, k, dtype=x2.dtype, device=x2.device) if out is None else out
    if m:
        nat.call("kab_rmsnorm", x2.data_ptr(), nat.dtype_code(x2), m, k, x2.stride(0), w.data_ptr(), float(eps),
                 h.data_ptr(), nat.stream_of(x2))
    return h


def rmsnorm_fp8(x: torch.Tensor, weight: torch.Tensor, eps: float, mx: bool = False, blocked: bool = False,
                out: torch.Tensor | None = None):
    """``(codes, scales)`` of ``RMSNorm(x) * weight`` (triton_fp8_producers.py:191-202): per
    token e4m3 (fp32 scales ``[rows]``) or MXFP8 with ``mx`` (e8m0 bytes ``[rows, K / 32]``,
    swizzled with ``blocked``); ``out``: also the norm's output."""
    nat.require_cuda(x, weight)
    x2 = q._rows(q._input(x))
    m, k = x2.shape
    if k > 16384 or k % (q.MX_BLOCK if mx else 8):  # the two passes (the fused kernel's row limit)
        h = _rmsnorm(x, weight, eps, out)
        return quantize_rows(h, mx=mx, blocked=blocked)
    w = weight.to(device=x2.device, dtype=x2.dtype).reshape(-1).contiguous()
    if w.numel() != k:
        raise ValueError(f"weight has {w.numel()} elements, expected {k}")
    _check_out(out, x2)
    if mx:
        codes, scales = q._mx_outputs(m, k, x2.device, blocked)
    else:
        codes = torch.empty(m, k, dtype=torch.float8_e4m3fn, device=x2.device)
        scales = torch.empty(m, dtype=torch.float32, device=x2.device)
    if m:  # one pass: the norm kept in registers and quantised (kab_rmsnorm_quant_fp8)
        nat.call("kab_rmsnorm_quant_fp8", x2.data_ptr(), nat.dtype_code(x2), m, k, x2.stride(0), w.data_ptr(),
                 float(eps), int(mx), int(mx and blocked), codes.data_ptr(), scales.data_ptr(), nat.ptr(out),
                 nat.stream_of(x2))
    return codes, scales


def rmsnorm_fp4(x: torch.Tensor, weight: torch.Tensor, eps: float, mx: bool = False, swizzle: bool = False,
                out: torch.Tensor | None = None, unbiased: bool = False):
    """``(codes, scales, outer)`` of ``RMSNorm(x) * weight`` quantised to NVFP4 (MXFP4 with
    ``mx``) (triton_fp4_producers.py:384-405); ``out``: also the norm's output; ``unbiased``:
    and the epilogue's per-token scale (fourth)."""
    fmt = _fp4_block(x.shape[-1], mx)
    nat.require_cuda(x, weight)
    x2 = q._rows(q._input(x))
    m, k = x2.shape
    if x2.dtype == torch.float32:  # the two passes (the fused kernel takes bf16 and fp16)
        h = _rmsnorm(x, weight, eps, out)
        return _result_fp4(h, q._fp4(h, fmt, nat.KAB_FP4_TOKEN, swizzle=swizzle), fmt, swizzle, unbiased)
    w = weight.to(device=x2.device, dtype=x2.dtype).reshape(-1).contiguous()
    if w.numel() != k:
        raise ValueError(f"weight has {w.numel()} elements, expected {k}")
    _check_out(out, x2)
    # one pass (kab_rmsnorm_quant_fp4); the bias correction reads h, so it is then written
    h = out if out is not None or not unbiased else torch.empty(m, k, dtype=x2.dtype, device=x2.device)
    res = q._fp4(x2, fmt, nat.KAB_FP4_TOKEN, swizzle=swizzle, h=h, norm=(w, eps))
    return _result_fp4(h, res, fmt, swizzle, unbiased) if unbiased else res
