"""Fused quantise producers, the GPU counterparts of kernel-agent's example producers
(``src/kernel_agent/agent/examples/triton_fp8_producers.py:177-222`` and
``triton_fp4_producers.py:369-434``): ``silu(gate) * up`` (or a plain row) quantised in the
producer's epilogue, so the next GEMM reads one byte (FP8) or half a byte (FP4) per
activation and no bf16 intermediate is written.

The values quantised are eager's (``F.silu`` rounded to the input dtype, the product
rounded again); codes and scales equal ``quant.quantize_*`` of those values bit for bit.
``out`` (optional, ``[rows, K]`` in the input dtype) also receives ``silu(gate) * up``.
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


def quantize_rows_fp4(x: torch.Tensor, mx: bool = False, swizzle: bool = False):
    """``(codes, scales, outer)`` of ``x [..., K]`` (triton_fp4_producers.py:369-381): NVFP4
    (per-token outer scale) or MXFP4 with ``mx``; scales row-major or swizzled."""
    nat.require_cuda(x)
    fmt = "mxfp4" if mx else "nvfp4"
    block = q.FP4_FORMATS[fmt][0]
    if x.shape[-1] % block:
        raise ValueError(f"the last dimension {x.shape[-1]} is not a multiple of the {fmt} block ({block})")
    return q._fp4(q._rows(q._input(x)), fmt, nat.KAB_FP4_TOKEN, swizzle=swizzle)


def silu_mul_fp4(gate: torch.Tensor, up: torch.Tensor | None = None, mx: bool = False,
                 swizzle: bool = False, out: torch.Tensor | None = None):
    """``(codes, scales, outer)`` of ``F.silu(gate) * up`` quantised to NVFP4 (MXFP4 with
    ``mx``) in the epilogue (triton_fp4_producers.py:408-434)."""
    nat.require_cuda(gate, up)
    g2, u2 = _split(gate, up)
    if g2.dtype not in (torch.bfloat16, torch.float16):
        raise ValueError("the fused SiLU * up producer takes bf16 or fp16")
    fmt = "mxfp4" if mx else "nvfp4"
    block = q.FP4_FORMATS[fmt][0]
    if g2.shape[1] % block:
        raise ValueError(f"the last dimension {g2.shape[1]} is not a multiple of the {fmt} block ({block})")
    _check_out(out, g2)
    return q._fp4(g2, fmt, nat.KAB_FP4_TOKEN, up=u2, swizzle=swizzle, h=out)
