"""GPU drop-in for ``kernel_agent.kernels.quant`` (kernel-agent 0.1.0,
``src/kernel_agent/kernels/quant.py``): the same names, arguments, return tuples, dtypes and
errors, computed by ``libkab.so`` on an sm_100a GPU.

Every function takes CUDA tensors (a CPU tensor raises ``ValueError("CUDA tensor
required")``: there is no CPU fallback) and returns new contiguous tensors on the input's
device, allocated through torch's caching allocator on the current stream (no host
synchronisation on the quantise paths, so they can be captured in a CUDA graph). Codes and
scales are bit for bit the reference's; the linears' outputs are the block-scaled fp32
products of the same codes (the tensor core's accumulation order) with the reference's
epilogue roundings.
"""

from __future__ import annotations

import ctypes
import math
import struct
from typing import Any

import torch

from .. import _native as nat
from . import gemm

# ------------------------------------------------------------------ constants (quant.py)

#: Largest finite value of each FP8 format (quant.py:98).
FP8_MAX = {torch.float8_e4m3fn: 448.0, torch.float8_e5m2: 57344.0}
#: e2m1 magnitudes of codes 0..7 (quant.py:189-190).
E2M1_VALUES = (0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0)
FP4_MAX = 6.0
#: Block-scaled FP4 formats (quant.py:194-197).
FP4_FORMATS: dict[str, tuple[int, torch.dtype]] = {
    "nvfp4": (16, torch.float8_e4m3fn),
    "mxfp4": (32, torch.float8_e8m0fnu),
}
#: MXFP8 block and scale rules (quant.py:464-474).
MX_BLOCK = 32
MX_RULES = ("ceil", "floor")
MX_SATURATION_SLACK = 2.0**-10
#: INT8 (quant.py:760-767).
INT8_MAX = 127.0
INT8_STEP = float(torch.tensor(1.0 / 127.0, dtype=torch.float32))
#: NVFP4 outer-scale step and granularities (quant.py:1033-1039).
NVFP4_OUTER_STEP = float(torch.tensor(1.0 / (FP4_MAX * 448.0), dtype=torch.float32))
FP4_GRANULARITIES = ("token", "tensor")
#: The NVFP4 scale-rule bounds (quant.py:1291-1296).
NVFP4_ROUNDING_RATIO = FP4_MAX * (1 + 2.0**-4)
FP4_SATURATION_SLACK = 2.0**-10
E4M3_MIN_NORMAL = 2.0**-6
NVFP4_STRESS_RATIOS = (
    *(1.1125 * 2.0**e for e in range(-6, 8)),
    *((k + 0.7) * 2.0**-9 for k in range(1, 6)),
)
#: The reference records torch._int_mm failures per device here (quant.py:851); this
#: package's INT8 GEMM is its own tcgen05 kernel and never falls back, so it stays empty.
INT_MM_FAILED: dict[tuple[str, str], str] = {}

_E4M3 = torch.float8_e4m3fn
_E8M0 = torch.float8_e8m0fnu
_RULE = {"ceil": 0, "floor": 1}


def _sig(value: float, digits: int = 4) -> float:
    return float(f"{value:.{digits}g}") if math.isfinite(value) else value


def _rows(x: torch.Tensor) -> torch.Tensor:
    """``x.reshape(-1, K)`` with unit stride along K and 16-byte aligned rows."""
    x2 = x.detach().reshape(-1, x.shape[-1]) if x.dim() != 2 else x.detach()
    if x2.stride(-1) != 1 or x2.stride(0) % 8 or x2.data_ptr() % 16:
        x2 = x2.contiguous()
    return x2


def _stream(t: torch.Tensor) -> int:
    return nat.stream_of(t)


def _input(x: torch.Tensor) -> torch.Tensor:
    """A floating-point input the kernels read (fp32, bf16 or fp16)."""
    if x.dtype not in nat.DTYPES:
        x = x.float()
    return x


def _amax(x2: torch.Tensor) -> torch.Tensor:
    """NaN-keeping max |x| (0-d fp32 on the device)."""
    out = torch.zeros((), dtype=torch.float32, device=x2.device)
    nat.call("kab_amax", x2.data_ptr(), nat.dtype_code(x2), x2.shape[0], x2.shape[1], x2.stride(0),
             out.data_ptr(), _stream(x2))
    return out


def _require_finite(x2: torch.Tensor) -> None:
    """quant.py:114-115: non-finite weights are refused (one device-to-host read)."""
    if x2.numel() and not math.isfinite(float(_amax(x2))):
        raise ValueError("the weight has non-finite values")


# ------------------------------------------------------------------ FP8 per token / channel


def quantize_fp8(
    weight: torch.Tensor, dtype: torch.dtype = torch.float8_e4m3fn
) -> tuple[torch.Tensor, torch.Tensor]:
    """quant.py:101-119: ``(q, scale)`` of a 2-D weight ``[out, in]``, one scale ``amax /
    448`` per output channel (1 for a zero row), e4m3 codes to nearest even."""
    if weight.dim() != 2:
        raise ValueError(f"expected a 2-D weight [out, in], got shape {tuple(weight.shape)}")
    if dtype not in FP8_MAX:
        raise ValueError(f"unsupported FP8 dtype {dtype}")
    if dtype != _E4M3:
        raise ValueError(f"unsupported FP8 dtype {dtype} (this build quantises to float8_e4m3fn)")
    nat.require_cuda(weight)
    w = _rows(_input(weight))
    _require_finite(w)
    return _fp8_rows(w)


def _fp8_rows(x2: torch.Tensor, up: torch.Tensor | None = None, h: torch.Tensor | None = None):
    m, k = x2.shape
    q = torch.empty(m, k, dtype=_E4M3, device=x2.device)
    s = torch.empty(m, dtype=torch.float32, device=x2.device)
    if m:
        nat.call("kab_quant_rows_fp8", x2.data_ptr(), nat.dtype_code(x2), m, k, x2.stride(0),
                 nat.ptr(up), 0 if up is None else up.stride(0), q.data_ptr(), s.data_ptr(),
                 nat.ptr(h), _stream(x2))
    return q, s


def quantize_fp8_activations(
    x: torch.Tensor, dtype: torch.dtype = torch.float8_e4m3fn
) -> tuple[torch.Tensor, torch.Tensor]:
    """quant.py:361-377: ``(q [tokens, in], scale [tokens])``, per token ``amax / 448``."""
    if dtype not in FP8_MAX:
        raise ValueError(f"unsupported FP8 dtype {dtype}")
    if dtype != _E4M3:
        raise ValueError(f"unsupported FP8 dtype {dtype} (this build quantises to float8_e4m3fn)")
    nat.require_cuda(x)
    return _fp8_rows(_rows(_input(x)))


def dequantize_fp8(q: torch.Tensor, scale: torch.Tensor, dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
    """quant.py:122-126: ``q * scale[:, None]`` (fp32 product, one rounding to ``dtype``)."""
    nat.require_cuda(q, scale)
    return (q.float() * scale.float()[:, None]).to(dtype)


# ------------------------------------------------------------------ INT8


def _smooth_of(smooth: torch.Tensor | None, k: int, device: torch.device) -> torch.Tensor | None:
    """quant.py:783-791."""
    if smooth is None:
        return None
    s = smooth.detach().float().to(device).reshape(-1).contiguous()
    if s.numel() != k:
        raise ValueError(f"expected {k} smoothing factors (one per input channel), got {s.numel()}")
    lo = _amax((-s).clamp_min(0).reshape(1, -1))  # > 0 when some factor is negative
    if not math.isfinite(float(_amax(s.reshape(1, -1)))) or float(lo) > 0 or bool((s == 0).any()):
        raise ValueError("smoothing factors must be finite and positive")
    return s


def _int8_rows(x2: torch.Tensor, smooth: torch.Tensor | None, mode: int):
    m, k = x2.shape
    q = torch.empty(m, k, dtype=torch.int8, device=x2.device)
    s = torch.empty(m, dtype=torch.float32, device=x2.device)
    if m:
        nat.call("kab_quant_rows_int8", x2.data_ptr(), nat.dtype_code(x2), m, k, x2.stride(0),
                 nat.ptr(smooth), mode if smooth is not None else 0, q.data_ptr(), s.data_ptr(),
                 _stream(x2))
    return q, s


def quantize_int8(weight: torch.Tensor, smooth: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """quant.py:794-813: per-output-channel int8 ``(q, scale)``, ``scale = amax * INT8_STEP``
    (1 for a zero row), codes ``round(w / scale)`` to nearest even, clamped to ±127; with
    ``smooth`` the weight is ``weight * smooth[None, :]``."""
    if weight.dim() != 2:
        raise ValueError(f"expected a 2-D weight [out, in], got shape {tuple(weight.shape)}")
    nat.require_cuda(weight)
    w = _rows(_input(weight))
    _require_finite(w)
    s = _smooth_of(smooth, w.shape[1], w.device)
    return _int8_rows(w, s, 2)


def quantize_int8_activations(x: torch.Tensor, smooth: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """quant.py:823-839: per-token int8 ``(q [tokens, in], scale [tokens])`` of ``x`` (of ``x /
    smooth`` with SmoothQuant factors)."""
    nat.require_cuda(x)
    x2 = _rows(_input(x))
    s = _smooth_of(smooth, x2.shape[1], x2.device)
    return _int8_rows(x2, s, 1)


def dequantize_int8(q: torch.Tensor, scale: torch.Tensor, dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
    """quant.py:816-820."""
    nat.require_cuda(q, scale)
    return (q.float() * scale.float()[:, None]).to(dtype)


# ------------------------------------------------------------------ MXFP8


def mx_scale_exponents(amax: torch.Tensor, rule: str = "ceil") -> torch.Tensor:
    """quant.py:479-495: the unbiased exponents (int32) of blocks with maxima ``amax``."""
    if rule not in MX_RULES:
        raise ValueError(f"unknown MXFP8 scale rule {rule!r} (one of {', '.join(MX_RULES)})")
    nat.require_cuda(amax)
    a = amax.detach().float().reshape(-1).contiguous()
    out = torch.empty(a.shape, dtype=torch.int32, device=a.device)
    if a.numel():
        nat.call("kab_mx_exponents", a.data_ptr(), a.numel(), _RULE[rule], out.data_ptr(), _stream(a))
    return out.reshape(amax.shape)


def mx_scale_values(scales: torch.Tensor) -> torch.Tensor:
    """quant.py:498-503."""
    if scales.dtype == torch.uint8:
        scales = scales.view(_E8M0)
    return scales.float()


def _mx_outputs(m: int, k: int, device, swizzle: bool):
    cols = k // MX_BLOCK
    if swizzle:
        size = -(-m // 128) * 128 * (-(-cols // 4)) * 4
        pad = m % 128 != 0 or cols % 4 != 0
        s = (torch.zeros if pad else torch.empty)(size, dtype=torch.uint8, device=device)
    else:
        s = torch.empty(m, cols, dtype=torch.uint8, device=device)
    return torch.empty(m, k, dtype=_E4M3, device=device), s


def _mxfp8(x2, rule: str, up=None, swizzle=False, h=None):
    m, k = x2.shape
    q, s = _mx_outputs(m, k, x2.device, swizzle)
    if m and k:
        nat.call("kab_quant_mxfp8", x2.data_ptr(), nat.dtype_code(x2), m, k, x2.stride(0),
                 nat.ptr(up), 0 if up is None else up.stride(0), _RULE[rule], q.data_ptr(),
                 s.data_ptr(), int(swizzle), nat.ptr(h), _stream(x2))
    return q, s


def quantize_mxfp8(x: torch.Tensor, rule: str = "ceil") -> tuple[torch.Tensor, torch.Tensor]:
    """quant.py:506-526: ``(codes e4m3 [rows, K], scales e8m0 [rows, K / 32])`` (unswizzled)."""
    k = x.shape[-1]
    if k % MX_BLOCK:
        raise ValueError(f"the last dimension {k} is not a multiple of the MXFP8 block (32)")
    if rule not in MX_RULES:
        raise ValueError(f"unknown MXFP8 scale rule {rule!r} (one of {', '.join(MX_RULES)})")
    nat.require_cuda(x)
    q, s = _mxfp8(_rows(_input(x)), rule)
    return q, s.view(_E8M0)


def dequantize_mxfp8(codes: torch.Tensor, scales: torch.Tensor, dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
    """quant.py:529-537."""
    nat.require_cuda(codes, scales)
    rows, k = codes.shape
    values = codes.float().reshape(rows, k // MX_BLOCK, MX_BLOCK)
    step = mx_scale_values(scales).reshape(rows, k // MX_BLOCK, 1)
    return (values * step).reshape(rows, k).to(dtype)


def mx_scale_offset(row: Any, col: Any, cols: int) -> Any:
    """quant.py:540-547: offset of scale ``[row, col]`` in the swizzled layout (ints or
    integer tensors)."""
    blocks_per_row = -(-cols // 4)
    block = (row // 128) * blocks_per_row + col // 4
    return block * 512 + (row % 32) * 16 + ((row % 128) // 32) * 4 + col % 4


def _swizzle(s: torch.Tensor) -> torch.Tensor:
    rows, cols = s.shape
    nrb, ncb = -(-rows // 128), -(-cols // 4)
    out = torch.zeros(nrb * 128 * ncb * 4, dtype=torch.uint8, device=s.device)
    if rows and cols:
        s = s.contiguous()
        nat.call("kab_swizzle_scales", s.data_ptr(), rows, cols, out.data_ptr(), _stream(s))
    return out


def swizzle_mx_scales(scales: torch.Tensor) -> torch.Tensor:
    """quant.py:550-564: ``[rows, K / 32]`` e8m0 / uint8 scales -> the flat 128 x 4 layout."""
    s = scales.view(torch.uint8) if scales.dtype == _E8M0 else scales
    if s.dtype != torch.uint8 or s.dim() != 2:
        raise ValueError(f"expected [rows, K / 32] e8m0 / uint8 scales, got {s.dtype} {s.shape}")
    nat.require_cuda(s)
    return _swizzle(s).view(_E8M0)


def swizzle_fp4_scales(scales: torch.Tensor) -> torch.Tensor:
    """quant.py:1176-1182: FP4 block scales -> the flat 128 x 4 layout, in their dtype."""
    nat.require_cuda(scales)
    return _swizzle(scales.view(torch.uint8)).view(scales.dtype)


# ------------------------------------------------------------------ FP4


def fp4_values(codes: torch.Tensor, scales: torch.Tensor) -> torch.Tensor:
    """quant.py:1110-1114: exact fp32 ``e2m1 * block scale`` ``[rows, K]``."""
    nat.require_cuda(codes, scales)
    rows, half = codes.shape
    k = 2 * half
    fmt = nat.KAB_NVFP4 if scales.dtype in (_E4M3, torch.uint8) and k // max(scales.shape[1], 1) == 16 else nat.KAB_MXFP4
    out = torch.empty(rows, k, dtype=torch.float32, device=codes.device)
    if rows and k:
        c, s = codes.contiguous(), scales.contiguous().view(torch.uint8)
        nat.call("kab_fp4_values", c.data_ptr(), s.data_ptr(), rows, k, fmt, out.data_ptr(), _stream(c))
    return out


def _fp4(x2, fmt: str, mode: int, amax=None, ts=None, up=None, swizzle=False, h=None, norm=None):
    """codes, scales and outer of x2 (or, with ``norm = (weight, eps)``, of its RMSNorm, in one
    pass by ``kab_rmsnorm_quant_fp4``; ``h`` then receives the norm's output)."""
    block, scale_dtype = FP4_FORMATS[fmt]
    m, k = x2.shape
    cols = k // block
    q = torch.empty(m, k // 2, dtype=torch.uint8, device=x2.device)
    if swizzle:
        size = -(-m // 128) * 128 * (-(-cols // 4)) * 4
        pad = m % 128 != 0 or cols % 4 != 0
        s = (torch.zeros if pad else torch.empty)(size, dtype=torch.uint8, device=x2.device)
    else:
        s = torch.empty(m, cols, dtype=torch.uint8, device=x2.device)
    outer = torch.empty(m, dtype=torch.float32, device=x2.device)
    if m and k and norm is not None:
        nat.call("kab_rmsnorm_quant_fp4", x2.data_ptr(), nat.dtype_code(x2), m, k, x2.stride(0),
                 norm[0].data_ptr(), float(norm[1]), nat.KAB_NVFP4 if fmt == "nvfp4" else nat.KAB_MXFP4,
                 int(swizzle), q.data_ptr(), s.data_ptr(), outer.data_ptr(), nat.ptr(h), _stream(x2))
    elif m and k:
        nat.call("kab_quant_fp4", x2.data_ptr(), nat.dtype_code(x2), m, k, x2.stride(0), nat.ptr(up),
                 0 if up is None else up.stride(0), nat.KAB_NVFP4 if fmt == "nvfp4" else nat.KAB_MXFP4,
                 mode, nat.ptr(amax), nat.ptr(ts), q.data_ptr(), s.data_ptr(), int(swizzle),
                 outer.data_ptr(), nat.ptr(h), _stream(x2))
    elif m:
        outer.fill_(1.0)
    return q, s.view(scale_dtype), outer


def quantize_fp4(
    weight: torch.Tensor, fmt: str = "nvfp4", unbiased: bool = False
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """quant.py:217-272: ``(codes [out, in / 2], scales [out, in / block], tensor_scale)``;
    NVFP4 ``tensor_scale = amax / (6 * 448)`` (a 0-d fp32 tensor), MXFP4 1."""
    if weight.dim() != 2:
        raise ValueError(f"expected a 2-D weight [out, in], got shape {tuple(weight.shape)}")
    if fmt not in FP4_FORMATS:
        raise ValueError(f"unknown FP4 format {fmt!r} (one of {', '.join(FP4_FORMATS)})")
    block, _ = FP4_FORMATS[fmt]
    rows, cols = weight.shape
    if cols % block:
        raise ValueError(f"in_features {cols} is not a multiple of the {fmt} block ({block})")
    nat.require_cuda(weight)
    w = _rows(_input(weight))
    amax = _amax(w)
    if w.numel() and not math.isfinite(float(amax)):
        raise ValueError("the weight has non-finite values")
    if fmt == "nvfp4":
        ts = torch.empty((), dtype=torch.float32, device=w.device)
        nat.call("kab_fp4_tensor_scale", amax.data_ptr(), ts.data_ptr(), _stream(w))
    else:
        ts = torch.ones((), dtype=torch.float32, device=w.device)
    q, s, _ = _fp4(w, fmt, nat.KAB_FP4_WEIGHT, ts=ts)
    if unbiased:  # quant.py:270-271: one factor per output channel, in the tensor scale's place
        ts = ts * fp4_bias_correction(w, q, s, ts)
    return q, s, ts


def quantize_fp4_activations(
    x: torch.Tensor, fmt: str = "nvfp4", granularity: str = "token"
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """quant.py:1056-1107: ``(codes [rows, K / 2], scales [rows, K / block], outer [rows])``."""
    if fmt not in FP4_FORMATS:
        raise ValueError(f"unknown FP4 format {fmt!r} (one of {', '.join(FP4_FORMATS)})")
    if granularity not in FP4_GRANULARITIES:
        raise ValueError(f"unknown granularity {granularity!r} ({', '.join(FP4_GRANULARITIES)})")
    block, _ = FP4_FORMATS[fmt]
    k = x.shape[-1]
    if k % block:
        raise ValueError(f"the last dimension {k} is not a multiple of the {fmt} block ({block})")
    nat.require_cuda(x)
    x2 = _rows(_input(x))
    if fmt == "nvfp4" and granularity == "tensor":
        return _fp4(x2, fmt, nat.KAB_FP4_TENSOR, amax=_amax(x2))
    return _fp4(x2, fmt, nat.KAB_FP4_TOKEN)


def dequantize_fp4(codes, scales, tensor_scale, dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
    """quant.py:275-294: ``e2m1 * scale * tensor_scale`` in fp32, one rounding to ``dtype``."""
    v = fp4_values(codes, scales)
    ts = torch.as_tensor(tensor_scale, dtype=torch.float32, device=v.device)
    ts = ts.reshape(()) if ts.numel() == 1 else ts.reshape(-1, 1)
    return (v * ts).to(dtype)


# ------------------------------------------------------------------ linears (tcgen05 GEMMs)


def int8_matmul(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """quant.py:854-885: exact int32 ``a [M, K] @ b [N, K]ᵀ`` (tcgen05 kind::i8)."""
    if a.dtype != torch.int8 or b.dtype != torch.int8 or a.dim() != 2 or b.dim() != 2:
        raise ValueError("int8_matmul takes 2-D int8 a [M, K] and b [N, K]")
    if a.shape[1] != b.shape[1]:
        raise ValueError(f"K differs: a {tuple(a.shape)}, b {tuple(b.shape)}")
    nat.require_cuda(a)
    b = b.to(a.device)
    if a.shape[0] == 0:
        return torch.zeros(0, b.shape[0], dtype=torch.int32, device=a.device)
    return gemm.int8(a, b)


def _linear_out(y: torch.Tensor, x: torch.Tensor, n: int) -> torch.Tensor:
    if y.dtype != x.dtype:
        y = y.to(x.dtype)
    return y.reshape(*x.shape[:-1], n)


def int8_w8a8_linear(
    x: torch.Tensor,
    q: torch.Tensor,
    scale: torch.Tensor,
    bias: torch.Tensor | None = None,
    *,
    smooth: torch.Tensor | None = None,
) -> torch.Tensor:
    """quant.py:901-923: per-token int8 activations, exact int32 products (tcgen05 kind::i8),
    ``acc * x_scale[m] * w_scale[n] (+ bias)`` in fp32 with one rounding to ``x``'s dtype:
    bit for bit the reference's result."""
    nat.require_cuda(x, q)
    xq, xs = quantize_int8_activations(x, smooth)
    y = gemm.int8(xq, q, xs, scale, bias, out_dtype=x.dtype)
    return _linear_out(y, x, q.shape[0])


def fp8_w8a8_linear(
    x: torch.Tensor,
    q: torch.Tensor,
    scale: torch.Tensor,
    bias: torch.Tensor | None = None,
) -> torch.Tensor:
    """quant.py:390-417: per-token e4m3 activations, e4m3 weight per channel, fp32
    accumulation (tcgen05 kind::f8f6f4), both scales and the bias in the epilogue."""
    nat.require_cuda(x, q)
    xq, xs = quantize_fp8_activations(x, q.dtype)
    y = gemm.fp8(xq, q, xs, scale, bias, out_dtype=x.dtype)
    return _linear_out(y, x, q.shape[0])


def _swizzled(scales: torch.Tensor, rows: int, cols: int) -> torch.Tensor:
    """Block scales in the swizzled layout: as given when already flat (1-D), else swizzled."""
    s = scales.view(torch.uint8) if scales.dtype != torch.uint8 else scales
    if s.dim() == 1:
        need = -(-rows // 128) * 128 * (-(-cols // 4)) * 4
        if s.numel() != need:
            raise ValueError(f"swizzled scales have {s.numel()} bytes, expected {need}")
        return s.contiguous()
    if tuple(s.shape) != (rows, cols):
        raise ValueError(f"expected scales [{rows}, {cols}], got {tuple(s.shape)}")
    return _swizzle(s)


def mxfp8_linear(
    x: torch.Tensor,
    q: torch.Tensor,
    scales: torch.Tensor,
    bias: torch.Tensor | None = None,
    *,
    rule: str = "ceil",
) -> torch.Tensor:
    """quant.py:581-620: ``x`` quantised to MXFP8 (scales written swizzled), the block-scaled
    GEMM (tcgen05 kind::mxf8f6f4, e8m0 per 32 on both operands) with a bf16 result, ``+ bias``
    in bf16, then ``x``'s dtype. ``scales``: the weight's ``[N, K / 32]`` (or already
    swizzled, flat)."""
    nat.require_cuda(x, q)
    k = x.shape[-1]
    if k % MX_BLOCK:
        raise ValueError(f"the last dimension {k} is not a multiple of the MXFP8 block (32)")
    xq, xs = _mxfp8(_rows(_input(x)), rule, swizzle=True)
    ws = _swizzled(scales, q.shape[0], k // MX_BLOCK)
    y = gemm.mxf8(xq, xs, q, ws, bias, out_dtype=torch.bfloat16)
    return _linear_out(y, x, q.shape[0])


def hadamard(n: int, device: torch.device | str | None = None) -> torch.Tensor:
    """quant.py:1150-1159: the orthonormal Sylvester-Hadamard matrix of order ``n`` (a power of
    two), fp32."""
    if n < 1 or n & (n - 1):
        raise ValueError(f"the Hadamard order must be a power of two, got {n}")
    h = torch.ones(1, 1, device=device)
    while h.shape[0] < n:
        h = torch.cat([torch.cat([h, h], 1), torch.cat([h, -h], 1)], 0)
    return h / math.sqrt(n)


def hadamard_rotate(x: torch.Tensor, block: int) -> torch.Tensor:
    """quant.py:1162-1173: ``x [..., K]`` with every ``block`` consecutive elements along K
    multiplied by ``hadamard(block)``, fp32 (one GPU pass: butterflies in shared memory)."""
    k = x.shape[-1]
    if k % block:
        raise ValueError(f"the last dimension {k} is not a multiple of the rotation ({block})")
    if block < 1 or block & (block - 1):
        raise ValueError(f"the Hadamard order must be a power of two, got {block}")
    nat.require_cuda(x)
    x2 = _rows(_input(x))
    out = torch.empty(x2.shape[0], k, dtype=torch.float32, device=x2.device)
    if x2.shape[0] and k:
        nat.call("kab_hadamard_rotate", x2.data_ptr(), nat.dtype_code(x2), x2.shape[0], k, x2.stride(0), block,
                 out.data_ptr(), _stream(x2))
    return out.reshape(*x.shape[:-1], k)


def _bias_correction(x2, codes, scales, fmt: str, outer, swizzled: bool) -> torch.Tensor:
    rows, k = x2.shape
    out = torch.empty(rows, dtype=torch.float32, device=x2.device)
    o, per_row = None, 0
    if outer is not None:
        o = torch.as_tensor(outer).detach().float().to(x2.device).reshape(-1).contiguous()
        per_row = int(o.numel() == rows and rows != 1)
        if o.numel() not in (1, rows):
            raise ValueError(f"expected an outer scale per row ([{rows}]) or one, got {o.numel()}")
    if rows:
        nat.call("kab_fp4_bias_correction", x2.data_ptr(), nat.dtype_code(x2), rows, k, x2.stride(0),
                 codes.contiguous().data_ptr(), scales.view(torch.uint8).contiguous().data_ptr(),
                 nat.KAB_NVFP4 if fmt == "nvfp4" else nat.KAB_MXFP4, int(swizzled), nat.ptr(o), per_row,
                 out.data_ptr(), _stream(x2))
    return out


def fp4_bias_correction(x: torch.Tensor, codes: torch.Tensor, scales: torch.Tensor,
                        outer: torch.Tensor | float | None = None) -> torch.Tensor:
    """quant.py:1117-1148: per row of ``x [rows, K]`` quantised to ``(codes, scales [rows, K /
    block] unswizzled, outer)``, ``c = sum x^2 / sum x x^`` (float64 sums; 1 where ``sum x x^``
    is not positive), fp32 ``[rows]`` (one GPU pass)."""
    nat.require_cuda(x, codes)
    x2 = _rows(_input(x))
    k = x2.shape[1]
    fmt = "nvfp4" if scales.shape[-1] * 16 == k else "mxfp4"
    if scales.dim() != 2 or scales.shape[-1] * FP4_FORMATS[fmt][0] != k:
        raise ValueError(f"expected unswizzled scales [rows, K / block] for K = {k}, got {tuple(scales.shape)}")
    return _bias_correction(x2, codes, scales, fmt, outer, swizzled=False)


def fp4_w4a4_linear(
    x: torch.Tensor,
    codes: torch.Tensor,
    scales: torch.Tensor,
    tensor_scale: torch.Tensor | float,
    bias: torch.Tensor | None = None,
    *,
    fmt: str = "nvfp4",
    granularity: str = "token",
    rotate: int | None = None,
    unbiased: bool = False,
) -> torch.Tensor:
    """quant.py:1201-1257: ``x`` quantised per call (block scales written swizzled; NVFP4's
    outer scale per token or per call, MXFP4's 1), the block-scaled GEMM (tcgen05
    kind::mxf4nvf4: e4m3 scales per 16 or e8m0 per 32 applied by the tensor core, fp32
    accumulation), then ``acc * (outer[m] * tensor_scale) (+ bias)`` in fp32 and one rounding
    to ``x``'s dtype. ``scales``: the weight's ``[N, K / block]`` (or already swizzled, flat,
    when K is a multiple of 256)."""
    if fmt not in FP4_FORMATS:
        raise ValueError(f"unknown FP4 format {fmt!r} (one of {', '.join(FP4_FORMATS)})")
    if granularity not in FP4_GRANULARITIES:
        raise ValueError(f"unknown granularity {granularity!r} ({', '.join(FP4_GRANULARITIES)})")
    nat.require_cuda(x, codes)
    block = FP4_FORMATS[fmt][0]
    k = x.shape[-1]
    if k % block:
        raise ValueError(f"the last dimension {k} is not a multiple of the {fmt} block ({block})")
    n = codes.shape[0]
    x2 = hadamard_rotate(_rows(_input(x)), rotate) if rotate else _rows(_input(x))
    kp = k + (-k % 256)  # the GEMM's k-step: zero codes and scales pad K (they add nothing)
    ws = scales
    if kp != k:
        if scales.dim() != 2:
            raise ValueError(f"K = {k} needs padding to {kp}: pass the unswizzled [N, K / {block}] scales")
        x2 = torch.nn.functional.pad(x2, (0, kp - k))
        codes = torch.nn.functional.pad(codes.view(torch.uint8), (0, (kp - k) // 2))
        ws = torch.nn.functional.pad(scales.view(torch.uint8), (0, (kp - k) // block))
    odt = x.dtype if x.dtype in (torch.bfloat16, torch.float16, torch.float32) else torch.float32
    ts = torch.as_tensor(tensor_scale, dtype=torch.float32, device=x2.device)
    if fmt == "nvfp4":
        mode = nat.KAB_FP4_TENSOR if granularity == "tensor" else nat.KAB_FP4_TOKEN
        amax = _amax(x2) if granularity == "tensor" else None
        xq, xs, outer = _fp4(x2, "nvfp4", mode, amax=amax, swizzle=True)
        if unbiased:  # quant.py:1231-1232: the activations' factor in the epilogue's outer scale
            outer = outer * _bias_correction(x2, xq, xs, "nvfp4", outer, swizzled=True)
        y = gemm.nvf4(xq, xs.view(torch.uint8), outer, codes, _swizzled(ws, n, kp // 16), ts, bias, out_dtype=odt)
    else:  # MXFP4: e8m0 scales per 32, outer 1 (quant.py:1079-1087)
        xq, xs, outer = _fp4(x2, "mxfp4", nat.KAB_FP4_TOKEN, swizzle=True)
        outer = outer * _bias_correction(x2, xq, xs, "mxfp4", outer, swizzled=True) if unbiased else None
        y = gemm.mxf4(xq, xs.view(torch.uint8), codes, _swizzled(ws, n, kp // 32), ts, bias, out_dtype=odt,
                      a_outer=outer)
    return _linear_out(y, x, n)


# ------------------------------------------------------------------ scale-rule checks (GPU reductions)


def _check_result(out: torch.Tensor) -> "nat.KabScaleCheck":
    host = out.cpu()  # one device-to-host read of the counts
    return nat.KabScaleCheck.from_buffer_copy(bytes(host.numpy().tobytes()))


def _worst(res) -> float:
    return struct.unpack("<f", struct.pack("<I", res.worst_ratio_bits))[0]


def mxfp8_saturation(x: torch.Tensor, scales: torch.Tensor) -> dict[str, Any]:
    """quant.py:623-660: how MXFP8 ``scales`` ``[rows, K / 32]`` (e8m0, uint8 biased exponents
    or values; unswizzled) fit the block maxima of ``x [..., K]``: ``blocks``, ``saturated``,
    ``share``, ``worst_ratio``, ``coarser``, ``not_pow2`` (one GPU pass)."""
    k = x.shape[-1]
    x2 = _rows(_input(x)) if x.dim() else x
    rows, nblocks = x2.shape[0], k // MX_BLOCK
    if k % MX_BLOCK or tuple(scales.shape) != (rows, nblocks):
        raise ValueError(
            f"expected scales [{rows}, {nblocks}] (rows of x, K / 32, unswizzled) for x "
            f"{tuple(x.shape)}, got {tuple(scales.shape)}"
        )
    nat.require_cuda(x2)
    step = mx_scale_values(scales).to(x2.device).contiguous()
    out = torch.empty(ctypes.sizeof(nat.KabScaleCheck), dtype=torch.uint8, device=x2.device)
    nat.call("kab_mxfp8_saturation", x2.data_ptr(), nat.dtype_code(x2), rows, k, x2.stride(0) if rows else k,
             step.data_ptr(), out.data_ptr(), _stream(x2))
    res = _check_result(out)
    blocks = rows * nblocks
    return {
        "blocks": blocks,
        "saturated": int(res.saturated),
        "share": _sig(res.saturated / blocks) if blocks else 0.0,
        "worst_ratio": _sig(_worst(res)) if blocks else 0.0,
        "coarser": int(res.coarser),
        "not_pow2": int(res.not_pow2),
    }


def mxfp8_scale_problem(x: torch.Tensor, scales: torch.Tensor) -> str | None:
    """quant.py:663-680: why ``scales`` are not a valid MXFP8 quantisation of ``x``; None when
    they are."""
    found = mxfp8_saturation(x, scales)
    if found["saturated"]:
        return (
            f"{found['saturated']} of {found['blocks']} MXFP8 blocks ({found['share']:.1%}) "
            f"saturate: block maximum up to {found['worst_ratio']:.4g} x scale, above e4m3's "
            "448 (their largest elements are clamped). Use the scale 2^ceil(log2(amax / 448)); "
            "the OCP rule 2^(floor(log2 amax) - 8) saturates maxima in (448, 512) x scale"
        )
    if found["not_pow2"]:
        return (
            f"{found['not_pow2']} of {found['blocks']} MXFP8 scales are not powers of two "
            "(ue8m0 holds an exponent only)"
        )
    return None


def _stress_blocks(rows: int, nb: int, block: int, seed: int) -> torch.Tensor:
    """Gaussian blocks ``[rows, nb, block]`` scaled so that each block's largest magnitude is
    1, at its largest Gaussian value (the stress inputs' shape, from a CPU generator)."""
    gen = torch.Generator().manual_seed(seed)
    v = torch.randn(rows, nb, block, generator=gen)
    peak = v.abs().argmax(dim=-1, keepdim=True)
    return v / v.abs().gather(-1, peak)


def mxfp8_stress_input(shape, *, dtype: torch.dtype = torch.bfloat16, device="cpu", seed: int = 0) -> torch.Tensor:
    """quant.py:683-704: blocks of 32 with maxima at ±1.9 x 2^e, e from -8 to 8 across blocks
    (the OCP floor rule saturates every block, the ceil rule none)."""
    k = int(shape[-1])
    if k % MX_BLOCK:
        raise ValueError(f"the last dimension {k} is not a multiple of the MXFP8 block (32)")
    rows = math.prod(int(n) for n in shape[:-1])
    v = _stress_blocks(rows, k // MX_BLOCK, MX_BLOCK, seed)
    e = torch.arange(rows * (k // MX_BLOCK)).reshape(rows, k // MX_BLOCK, 1) % 17 - 8
    v = v * 1.9 * torch.pow(2.0, e.float())
    return v.reshape(*shape).to(dtype=dtype, device=device)


def fp4_format_of(k: int, scales: torch.Tensor) -> str:
    """quant.py:1300-1316: the FP4 format of activation scales for ``K`` = ``k``."""
    if scales.dtype == torch.float8_e4m3fn:
        return "nvfp4"
    if scales.dtype == torch.float8_e8m0fnu:
        return "mxfp4"
    width = scales.shape[-1] if scales.dim() == 2 else -1
    for fmt, (block, _) in FP4_FORMATS.items():
        if k % block == 0 and width == k // block:
            return fmt
    raise ValueError(
        f"expected FP4 activation scales [rows, K / 16] (NVFP4, e4m3) or [rows, K / 32] (MXFP4, "
        f"e8m0), unswizzled, for K = {k}; got {scales.dtype} {tuple(scales.shape)}"
    )


def fp4_scale_values(scales: torch.Tensor, fmt: str) -> torch.Tensor:
    """quant.py:1319-1324: fp32 values of FP4 block scales."""
    if scales.dtype == torch.uint8:
        scales = scales.view(FP4_FORMATS[fmt][1])
    return scales.float()


def _fp4_block_check(x: torch.Tensor, scales: torch.Tensor, outer, fmt: str | None):
    """One GPU pass of the W4A4 scale-rule check: (its raw counts, the number of blocks, fmt)."""
    k = x.shape[-1]
    x2 = _rows(_input(x))
    rows = x2.shape[0]
    fmt = fmt or fp4_format_of(k, scales)
    block = FP4_FORMATS[fmt][0]
    nb = k // block if k % block == 0 else -1
    if nb < 0 or tuple(scales.shape) != (rows, nb):
        raise ValueError(
            f"expected {fmt} scales [{rows}, {max(nb, 0)}] (rows of x, K / {block}, unswizzled) "
            f"for x {tuple(x.shape)}, got {tuple(scales.shape)}"
        )
    nat.require_cuda(x2)
    s = fp4_scale_values(scales, fmt).to(x2.device).contiguous()
    if outer is None:
        o, per_row = None, 0
    else:
        o = torch.as_tensor(outer).detach().float().to(x2.device).reshape(-1).contiguous()
        if o.numel() == 1:
            per_row = 0
        elif o.numel() == rows:
            per_row = 1
        else:
            raise ValueError(f"expected an outer scale per row ([{rows}]) or one, got {o.numel()}")
    out = torch.empty(ctypes.sizeof(nat.KabScaleCheck), dtype=torch.uint8, device=x2.device)
    nat.call("kab_fp4_scale_check", x2.data_ptr(), nat.dtype_code(x2), rows, k, x2.stride(0) if rows else k,
             nat.KAB_NVFP4 if fmt == "nvfp4" else nat.KAB_MXFP4, s.data_ptr(), nat.ptr(o), per_row,
             out.data_ptr(), _stream(x2))
    return _check_result(out), rows * nb, fmt


def fp4_scale_check(x: torch.Tensor, scales: torch.Tensor, outer: torch.Tensor | float | None = None,
                    fmt: str | None = None) -> dict[str, Any]:
    """quant.py:1325-1416: how W4A4 activation block scales (unswizzled) fit the block maxima
    of ``x`` with the given outer scale: ``format``, ``blocks``, ``saturated``, ``share``,
    ``worst_ratio``, ``underflow``, ``nonfinite``, ``not_representable``, ``coarser`` (one
    GPU pass)."""
    res, blocks, fmt = _fp4_block_check(x, scales, outer, fmt)
    return {
        "format": fmt,
        "blocks": blocks,
        "saturated": int(res.saturated),
        "share": _sig(res.saturated / blocks) if blocks else 0.0,
        "worst_ratio": _sig(_worst(res)) if blocks else 0.0,
        "underflow": int(res.underflow),
        "nonfinite": int(res.nonfinite),
        "not_representable": int(res.not_representable),
        "coarser": int(res.coarser),
    }


def fp4_scale_problem(x: torch.Tensor, scales: torch.Tensor, outer: torch.Tensor | float | None = None,
                      fmt: str | None = None) -> str | None:
    """quant.py:1419-1457: why ``(scales, outer)`` are not a valid W4A4 activation
    quantisation of ``x``; None when they are."""
    found = fp4_scale_check(x, scales, outer, fmt)
    blocks, fmt = found["blocks"], found["format"]
    if found["nonfinite"]:
        return (
            f"{found['nonfinite']} of {blocks} {fmt} blocks have a scale or an outer scale that "
            "is not finite, or an outer scale <= 0"
        )
    if found["saturated"] and fmt == "nvfp4":
        return (
            f"{found['saturated']} of {blocks} NVFP4 blocks ({found['share']:.1%}) saturate "
            f"beyond the rounding of their e4m3 scale: block maximum up to "
            f"{found['worst_ratio']:.4g} x step (scale x outer), above {NVFP4_ROUNDING_RATIO:g} "
            "(6 x (1 + e4m3's half step)); round the block scale bmax / (outer x 6) to "
            "nearest (or up), never down, and keep the outer scale at amax / (6 x 448) per "
            "row or per call so that no block scale clamps at 448"
        )
    if found["saturated"]:
        return (
            f"{found['saturated']} of {blocks} MXFP4 blocks ({found['share']:.1%}) saturate: "
            f"block maximum up to {found['worst_ratio']:.4g} x scale, above e2m1's 6 (their "
            "largest elements are clamped). Use the scale 2^ceil(log2(amax / 6)); the OCP rule "
            "2^(floor(log2 amax) - 2) saturates maxima in (6, 8) x scale"
        )
    if found["underflow"]:
        return (
            f"{found['underflow']} of {blocks} NVFP4 blocks with a non-zero maximum got block "
            "scale 0 where e4m3 rounding to nearest gives a non-zero (subnormal, 2^-9 steps) "
            "scale: all their codes are 0 (subnormal scales flushed to zero?)"
        )
    if found["not_representable"]:
        what = "e4m3 values" if fmt == "nvfp4" else "powers of two (e8m0 holds an exponent only)"
        return f"{found['not_representable']} of {blocks} {fmt} block scales are not {what}"
    return None


def fp4_stress_input(shape, fmt: str = "nvfp4", *, dtype: torch.dtype = torch.bfloat16, device="cpu",
                     seed: int = 0) -> torch.Tensor:
    """quant.py:1467-1508: activations on which saturating W4A4 scale rules show (NVFP4: the
    row maximum 64 in each row's first block, the other blocks' maxima 64 x m / 448 for m of
    ``NVFP4_STRESS_RATIOS``; MXFP4: :func:`mxfp8_stress_input`)."""
    if fmt == "mxfp4":
        return mxfp8_stress_input(shape, dtype=dtype, device=device, seed=seed)
    if fmt != "nvfp4":
        raise ValueError(f"unknown FP4 format {fmt!r} (one of {', '.join(FP4_FORMATS)})")
    block = FP4_FORMATS[fmt][0]
    k = int(shape[-1])
    if k % block:
        raise ValueError(f"the last dimension {k} is not a multiple of the NVFP4 block (16)")
    rows, nb = math.prod(int(n) for n in shape[:-1]), k // block
    v = _stress_blocks(rows, nb, block, seed)
    targets = torch.tensor(NVFP4_STRESS_RATIOS)
    index = torch.arange(rows * nb).reshape(rows, nb) % len(NVFP4_STRESS_RATIOS)
    bmax = 64.0 * targets[index] / 448.0
    bmax[:, 0] = 64.0
    return (v * bmax[..., None]).reshape(*shape).to(dtype=dtype, device=device)


# ------------------------------------------------------------------ error reports (GPU reductions)


def _pair_stats(x: torch.Tensor, y: torch.Tensor) -> torch.Tensor:
    """Per-row float64 sums of a pair ``x``, ``y`` ``[rows, k]`` in one GPU pass
    (``kab_row_pair_stats``): columns sum x^2, sum y^2, sum (x - y)^2, sum x y, max |x|,
    count x != 0, count (x != 0 and y == 0), max |y|."""
    def two_d(t: torch.Tensor) -> torch.Tensor:
        t = t if t.dtype in nat.DTYPES else t.float()
        t = t.reshape(-1, t.shape[-1])
        return t if t.stride(-1) == 1 else t.contiguous()

    x2, y2 = two_d(x), two_d(y)
    if x2.shape != y2.shape:
        raise ValueError(f"shapes differ: {tuple(x2.shape)} and {tuple(y2.shape)}")
    nat.require_cuda(x2, y2)
    rows, k = x2.shape
    out = torch.empty(rows, 8, dtype=torch.float64, device=x2.device)
    if rows:
        nat.call("kab_row_pair_stats", x2.data_ptr(), nat.dtype_code(x2), x2.stride(0) if k else 1, y2.data_ptr(),
                 nat.dtype_code(y2), y2.stride(0) if k else 1, rows, k, out.data_ptr(), _stream(x2))
    return out


def _weight_fields(st: torch.Tensor, k: int) -> dict[str, Any]:
    """quant.py:302-318: rel_l2, worst_channel_rel_l2, underflow and crest of a weight against
    its dequantised values, from the rows' pair sums."""
    tot = st.sum(dim=0)
    row_norm = st[:, 0].sqrt()
    live = row_norm > 0
    row_err = st[:, 2].sqrt() / row_norm.clamp_min(1e-30)
    crest = st[:, 4] / (row_norm / math.sqrt(max(k, 1))).clamp_min(1e-30)
    neg = torch.tensor(float("-inf"), dtype=torch.float64, device=st.device)
    vals = torch.stack([tot[0].sqrt(), tot[2].sqrt(), torch.where(live, row_err, neg).max() if st.shape[0] else neg,
                        tot[6], tot[5], torch.where(live, crest, neg).max() if st.shape[0] else neg]).tolist()
    norm, err, worst, flushed, nonzero, cr = vals
    return {
        "rel_l2": _sig(err / norm if norm > 0 else 0.0),
        "worst_channel_rel_l2": _sig(worst if norm > 0 else 0.0),
        "underflow": _sig(flushed / max(int(nonzero), 1)),
        "crest": _sig(cr if norm > 0 else 0.0),
    }


def _output_fields(ref: torch.Tensor, new: torch.Tensor) -> dict[str, float]:
    """quant.py:320-325 / 460-472: output_rel_l2, output_cosine, output_norm_ratio and
    output_gain of ``new`` against ``ref`` (fp32 outputs), from one pass of pair sums."""
    tot = _pair_stats(ref, new).sum(dim=0).tolist()
    ref_norm, new_norm, dot = math.sqrt(tot[0]), math.sqrt(tot[1]), tot[3]
    cos = dot / (ref_norm * new_norm) if ref_norm and new_norm else 1.0
    return {
        "output_rel_l2": _sig(math.sqrt(tot[2]) / ref_norm if ref_norm else 0.0),
        "output_cosine": round(cos, 6),
        "output_norm_ratio": round(new_norm / ref_norm, 5) if ref_norm else 1.0,
        "output_gain": round(dot / ref_norm**2, 5) if ref_norm else 1.0,
    }


def _activation_fields(a: torch.Tensor, a_hat: torch.Tensor, k: int) -> dict[str, float]:
    """quant.py:455-469: activation_rel_l2, activation_crest (largest amax / RMS of a token)
    and activation_underflow of the quantised activations."""
    st = _pair_stats(a, a_hat)
    tot = st.sum(dim=0)
    rms = (st[:, 0] / max(k, 1)).sqrt()
    crest = st[:, 4] / rms.clamp_min(1e-30)
    live = rms > 0
    neg = torch.tensor(float("-inf"), dtype=torch.float64, device=st.device)
    norm, err, cr, flushed, nonzero = torch.stack(
        [tot[0].sqrt(), tot[2].sqrt(), torch.where(live, crest, neg).max() if st.shape[0] else neg, tot[6],
         tot[5]]).tolist()
    return {
        "activation_rel_l2": _sig(err / norm if norm > 0 else 0.0),
        "activation_crest": _sig(cr if cr != float("-inf") else 0.0),
        "activation_underflow": _sig(flushed / max(int(nonzero), 1)),
    }


def _error_metrics(w: torch.Tensor, deq: torch.Tensor, x: torch.Tensor | None) -> dict[str, Any]:
    """quant.py:302-326: the weight report of ``deq`` against ``w`` (fp32 ``[out, in]``) and,
    with activations ``x``, the fp32 output error of ``x @ deqᵀ`` against ``x @ wᵀ``."""
    report = _weight_fields(_pair_stats(w, deq), w.shape[1])
    if x is not None:
        a = x.detach().float().reshape(-1, w.shape[1]).to(w.device)
        out = _output_fields(a @ w.T, a @ deq.T)
        report["output_rel_l2"] = out["output_rel_l2"]
        report["output_cosine"] = out["output_cosine"]
    return report


def fp8_error(weight: torch.Tensor, q: torch.Tensor, scale: torch.Tensor,
              x: torch.Tensor | None = None) -> dict[str, Any]:
    """quant.py:133-181: numerical error of ``weight`` stored as ``(q, scale)``: ``format``,
    ``granularity``, ``rel_l2``, ``worst_channel_rel_l2``, ``underflow``, ``crest``,
    ``bytes``; with ``x``: ``output_rel_l2`` and ``output_cosine`` (fp32 GEMMs)."""
    nat.require_cuda(weight, q)
    w = weight.detach().float()
    deq = dequantize_fp8(q, scale, torch.float32).to(w.device)
    return {
        "format": str(q.dtype).removeprefix("torch."),
        "granularity": "per output channel",
        **_error_metrics(w, deq, x),
        "bytes": {
            "before": weight.numel() * weight.element_size(),
            "after": q.numel() * q.element_size() + scale.numel() * scale.element_size(),
        },
    }


def _one(scale: torch.Tensor | float) -> bool:
    return not isinstance(scale, torch.Tensor) or scale.numel() == 1


def fp4_error(weight: torch.Tensor, codes: torch.Tensor, scales: torch.Tensor, tensor_scale: torch.Tensor | float,
              x: torch.Tensor | None = None) -> dict[str, Any]:
    """quant.py:328-359: :func:`fp8_error`'s report for ``weight`` stored as
    :func:`quantize_fp4`'s ``(codes, scales, tensor_scale)``."""
    nat.require_cuda(weight, codes)
    w = weight.detach().float()
    deq = dequantize_fp4(codes, scales, tensor_scale, torch.float32).to(w.device)
    fmt = next((f for f, (_, dtype) in FP4_FORMATS.items() if dtype == scales.dtype), "fp4")
    block = w.shape[1] // max(scales.shape[1], 1)
    kind = "e4m3 scale per {} + fp32 tensor scale" if fmt == "nvfp4" else "e8m0 scale per {}"
    tensor_scales = 1 if _one(tensor_scale) else torch.as_tensor(tensor_scale).numel()
    if tensor_scales > 1:
        kind += " x fp32 per channel (unbiased)"
    return {
        "format": fmt,
        "granularity": kind.format(block),
        **_error_metrics(w, deq, x),
        "bytes": {
            "before": weight.numel() * weight.element_size(),
            "after": codes.numel() + scales.numel() * scales.element_size() + 4 * tensor_scales,
        },
    }


def fp8_w8a8_error(weight: torch.Tensor, q: torch.Tensor, scale: torch.Tensor, x: torch.Tensor) -> dict[str, Any]:
    """quant.py:420-476: :func:`fp8_error` of the weight plus the per-token activations'
    ``activation_rel_l2`` / ``activation_crest`` / ``activation_underflow`` and the W8A8
    output's ``output_rel_l2`` / ``output_cosine`` / ``output_norm_ratio`` against
    ``x @ Wᵀ`` in fp32 (the W8A8 product on the tcgen05 kind::f8f6f4 GEMM, fp32 out)."""
    report = fp8_error(weight, q, scale)
    w = weight.detach().float()
    a = x.detach().float().reshape(-1, w.shape[1]).to(w.device)
    xq, xs = quantize_fp8_activations(a, q.dtype)
    a_hat = dequantize_fp8(xq, xs, torch.float32)
    out = _output_fields(a @ w.T, gemm.fp8(xq, q, xs, scale, None, out_dtype=torch.float32))
    report.update(activations="e4m3 per token", **_activation_fields(a, a_hat, w.shape[1]),
                  output_rel_l2=out["output_rel_l2"], output_cosine=out["output_cosine"],
                  output_norm_ratio=out["output_norm_ratio"])
    return report


def mxfp8_error(weight: torch.Tensor, q: torch.Tensor, scales: torch.Tensor, x: torch.Tensor | None = None,
                rule: str = "ceil") -> dict[str, Any]:
    """quant.py:707-768: the weight report of an MXFP8 layer and, with ``x`` (quantised with
    ``rule``), ``activation_rel_l2``, ``activation_saturation`` (share, worst_ratio) and the
    output error of the block-scaled GEMM (tcgen05 kind::mxf8f6f4, fp32 out) against
    ``x @ Wᵀ`` in fp32."""
    nat.require_cuda(weight, q)
    w = weight.detach().float()
    deq = dequantize_mxfp8(q, scales, torch.float32).to(w.device)
    report: dict[str, Any] = {
        "format": "mxfp8",
        "granularity": f"e4m3 + e8m0 scale per {MX_BLOCK} along K, both operands ({rule} rule)",
        **_error_metrics(w, deq, None),
        "bytes": {"before": weight.numel() * weight.element_size(), "after": q.numel() + scales.numel()},
    }
    if x is None:
        return report
    a = x.detach().float().reshape(-1, w.shape[1]).to(w.device)
    xq, xs = quantize_mxfp8(a, rule)
    a_hat = dequantize_mxfp8(xq, xs, torch.float32)
    if w.shape[1] % 128 == 0 and q.shape[0] % 128 == 0:  # the block-scaled GEMM's shapes
        new = gemm.mxf8(xq, _swizzle(xs.view(torch.uint8)), q,
                        _swizzled(scales, q.shape[0], w.shape[1] // MX_BLOCK), None, out_dtype=torch.float32)
    else:  # quant.py:745: the fp32 product of the dequantised operands
        new = a_hat @ deq.T
    out = _output_fields(a @ w.T, new)
    saturation = mxfp8_saturation(a, xs)
    return {
        **report,
        "activations": f"e4m3 + e8m0 per {MX_BLOCK} ({rule} rule)",
        "activation_rel_l2": _activation_fields(a, a_hat, w.shape[1])["activation_rel_l2"],
        "activation_saturation": {k: saturation[k] for k in ("share", "worst_ratio")},
        "output_rel_l2": out["output_rel_l2"],
        "output_cosine": out["output_cosine"],
        "output_norm_ratio": out["output_norm_ratio"],
    }


def int8_error(weight: torch.Tensor, q: torch.Tensor, scale: torch.Tensor,
               x: torch.Tensor | None = None) -> dict[str, Any]:
    """quant.py:926-949: :func:`fp8_error`'s report for ``weight`` stored as
    :func:`quantize_int8`'s ``(q, scale)``."""
    nat.require_cuda(weight, q)
    w = weight.detach().float()
    deq = dequantize_int8(q, scale, torch.float32).to(w.device)
    return {
        "format": "int8",
        "granularity": "per output channel, symmetric (amax / 127)",
        **_error_metrics(w, deq, x),
        "bytes": {
            "before": weight.numel() * weight.element_size(),
            "after": q.numel() + scale.numel() * scale.element_size(),
        },
    }


def int8_w8a8_error(weight: torch.Tensor, q: torch.Tensor, scale: torch.Tensor, x: torch.Tensor, *,
                    smooth: torch.Tensor | None = None) -> dict[str, Any]:
    """quant.py:951-1000: the weight report of :func:`int8_error` (of ``weight * smooth`` with
    SmoothQuant), the per-token activations' report and the INT8 W8A8 output (exact int32
    products on the tcgen05 kind::i8 GEMM, both scales in fp32) against ``x @ Wᵀ`` in fp32."""
    nat.require_cuda(weight, q)
    w = weight.detach().float()
    a = x.detach().float().reshape(-1, w.shape[1]).to(w.device)
    s = _smooth_of(smooth, w.shape[1], w.device)
    report = int8_error(w if s is None else w * s[None, :], q, scale)
    xq, xs = quantize_int8_activations(a, s)
    a_hat = xq.float() * xs[:, None]
    if s is not None:
        a_hat = a_hat * s[None, :]
    new = gemm.int8(xq, q.to(xq.device), xs, scale.float().to(xq.device), None, out_dtype=torch.float32)
    out = _output_fields(a @ w.T, new)
    report.update(activations="int8 per token" + (" (SmoothQuant)" if s is not None else ""),
                  **_activation_fields(a, a_hat, w.shape[1]), output_rel_l2=out["output_rel_l2"],
                  output_cosine=out["output_cosine"], output_norm_ratio=out["output_norm_ratio"])
    return report


def int8_weights_linear(x: torch.Tensor, q: torch.Tensor, scale: torch.Tensor,
                        bias: torch.Tensor | None = None) -> torch.Tensor:
    """quant.py:888-899: ``x @ Wᵀ + bias`` with INT8 weight-only numerics: the activations as
    they are, the int8 codes as values, fp32 accumulation (a plain fp32 GEMM), the
    per-channel scale (and the bias) once per output, one rounding to ``x``'s dtype."""
    nat.require_cuda(x, q)
    a = x.reshape(-1, x.shape[-1]).float()
    y = (a @ q.to(a.device).float().T) * scale.float().to(a.device)[None, :]
    if bias is not None:
        y = y + bias.float().to(a.device)
    return y.to(x.dtype).reshape(*x.shape[:-1], q.shape[0])


def smoothquant_factors(act_amax: torch.Tensor, weight: torch.Tensor, alpha: float = 0.5) -> torch.Tensor:
    """quant.py:1002-1041: SmoothQuant's per-input-channel factors ``s_j = amax(|X_j|)^alpha /
    amax(|W_j|)^(1 - alpha)`` (fp32 ``[in]``; 1 where either operand's channel is zero or the
    activation maximum is not finite), clamped to [1e-5, 1e5]."""
    a = act_amax.detach().float().reshape(-1)
    nat.require_cuda(a)
    w = weight.detach().float().abs().amax(dim=0).to(a.device)
    if a.numel() != w.numel():
        raise ValueError(f"{a.numel()} activation maxima for a weight with {w.numel()} inputs")
    if not 0.0 <= alpha <= 1.0:
        raise ValueError(f"alpha must be in [0, 1], got {alpha}")
    ok = (a > 0) & (w > 0) & torch.isfinite(a)
    s = a.clamp_min(1e-30).pow(alpha) / w.clamp_min(1e-30).pow(1.0 - alpha)
    return torch.where(ok, s.clamp(1e-5, 1e5), torch.ones_like(s)).contiguous()


def fp4_saturation(x: torch.Tensor, scales: torch.Tensor, outer: torch.Tensor, fmt: str = "nvfp4") -> dict[str, Any]:
    """quant.py:1260-1297: how FP4 activation scales fit the block maxima of ``x`` (one GPU
    pass of the scale check): ``blocks``, ``saturated`` (ratio above 6 x (1 + 2^-20)),
    ``share`` and ``worst_ratio``."""
    res, blocks, _ = _fp4_block_check(x, scales, outer, fmt)
    sat = int(res.saturated_plain)
    return {
        "blocks": blocks,
        "saturated": sat,
        "share": _sig(sat / blocks) if blocks else 0.0,
        "worst_ratio": _sig(_worst(res)) if blocks else 0.0,
    }


def fp4_w4a4_error(weight: torch.Tensor, codes: torch.Tensor, scales: torch.Tensor,
                   tensor_scale: torch.Tensor | float, x: torch.Tensor, *, fmt: str = "nvfp4",
                   granularity: str = "token", rotate: int | None = None, unbiased: bool = False) -> dict[str, Any]:
    """quant.py:1511-1573: the weight report of :func:`fp4_error` (of the rotated weight), the
    activations' ``activation_rel_l2`` / ``activation_crest`` / ``activation_saturation``, and
    the W4A4 output (the block-scaled tcgen05 GEMM with its fp32 epilogue) against
    ``x @ Wᵀ`` in fp32: ``output_rel_l2``, ``output_cosine``, ``output_norm_ratio``,
    ``output_gain``."""
    nat.require_cuda(weight, codes)
    w = weight.detach().float()
    a = x.detach().float().reshape(-1, w.shape[1]).to(w.device)
    report = fp4_error(hadamard_rotate(w, rotate) if rotate else w, codes, scales, tensor_scale)
    a_rot = hadamard_rotate(a, rotate) if rotate else a
    xq, xs, outer = quantize_fp4_activations(a_rot, fmt, granularity)
    saturation = fp4_saturation(a_rot, xs, outer, fmt)
    if unbiased:
        outer = outer * fp4_bias_correction(a_rot, xq, xs, outer)
    a_hat = fp4_values(xq, xs) * outer[:, None]
    act = _activation_fields(a_rot, a_hat, w.shape[1])
    crest = _activation_fields(a, a, w.shape[1])["activation_crest"]  # before the rotation
    new = fp4_w4a4_linear(a, codes, scales, tensor_scale, fmt=fmt, granularity=granularity, rotate=rotate,
                          unbiased=unbiased)
    out = _output_fields(a @ w.T, new)
    block, kind = FP4_FORMATS[fmt][0], "e4m3" if fmt == "nvfp4" else "e8m0"
    report.update(
        activations=f"{fmt}: e2m1 + {kind} scale per {block}"
        + (f" x fp32 per {granularity}" if fmt == "nvfp4" else "")
        + (f", Hadamard {rotate}" if rotate else "")
        + (", unbiased" if unbiased else ""),
        activation_rel_l2=act["activation_rel_l2"],
        activation_crest=crest,
        activation_saturation={k: saturation[k] for k in ("share", "worst_ratio")},
        **out,
    )
    return report


class _InputRecorder:
    """Records the first ``calls`` inputs of every ``nn.Linear`` of a module while it runs
    (forward pre-hooks, removed on exit), each as ``[rows, in_features]``."""

    def __init__(self, module: torch.nn.Module, calls: int):
        self.layers = {n: m for n, m in module.named_modules() if isinstance(m, torch.nn.Linear)}
        self.calls = calls
        self.inputs: dict[str, list[torch.Tensor]] = {}
        self._hooks: list[Any] = []

    def _hook_for(self, name: str):
        def record(_: torch.nn.Module, args: tuple[Any, ...]) -> None:
            got = self.inputs.setdefault(name, [])
            if len(got) < self.calls and isinstance(args[0], torch.Tensor):
                got.append(args[0].detach().reshape(-1, args[0].shape[-1]))
        return record

    def __enter__(self) -> "_InputRecorder":
        self._hooks = [m.register_forward_pre_hook(self._hook_for(n)) for n, m in self.layers.items()]
        return self

    def __exit__(self, *exc) -> None:
        for h in self._hooks:
            h.remove()

    def rows(self) -> dict[str, torch.Tensor]:
        """The recorded inputs of each layer that ran, concatenated, in module order."""
        return {n: torch.cat(self.inputs[n]) for n in self.layers if n in self.inputs}


def _same_values(a: torch.Tensor, b: torch.Tensor) -> bool:
    """quant.py:1656-1658: two layers read the same inputs (same shape, dtype, device and values)."""
    return a.shape == b.shape and a.dtype == b.dtype and a.device == b.device and torch.equal(a, b)


def _input_groups(inputs: dict[str, torch.Tensor]) -> dict[str, str]:
    """Each layer's group: the first layer (module order) that read the same inputs (q / k / v,
    gate / up), itself when none did."""
    leaders: list[tuple[str, torch.Tensor]] = []
    groups: dict[str, str] = {}
    for name, x in inputs.items():
        leader = next((lead for lead, y in leaders if _same_values(x, y)), None)
        if leader is None:
            leaders.append((name, x))
            leader = name
        groups[name] = leader
    return groups


def _sensitivity_of(layer: torch.nn.Linear, x: torch.Tensor, fmt: str, granularity: str,
                    rotate: int | None) -> dict[str, Any] | None:
    """One layer quantised alone to W4A4 and to FP8 W8A8 on inputs ``x``: its row (without
    name, group and FLOP share) and its GEMM FLOPs; None when W4A4 does not apply (K not a
    multiple of the block or of the rotation, or no inputs)."""
    w = layer.weight.detach()
    out_f, in_f = w.shape
    x = x.to(w.device)
    if in_f % (rotate or FP4_FORMATS[fmt][0]) or x.numel() == 0:
        return None
    codes, scales, ts = quantize_fp4(hadamard_rotate(w, rotate) if rotate else w, fmt)
    w4 = fp4_w4a4_error(w, codes, scales, ts, x, fmt=fmt, granularity=granularity, rotate=rotate)
    w8 = fp8_w8a8_error(w, *quantize_fp8(w), x)
    rows = int(x.shape[0])
    return {
        "rows": rows, "in_features": int(in_f), "out_features": int(out_f),
        "activation_crest": w4["activation_crest"],
        "w4a4_rel_l2": w4["output_rel_l2"],
        "w4a4_norm_change": _sig(w4["output_norm_ratio"] - 1.0),
        "fp8_rel_l2": w8["output_rel_l2"],
        "_flops": 2 * rows * int(in_f) * int(out_f),
    }


def fp4_w4a4_sensitivity(module: torch.nn.Module, run, *, fmt: str = "nvfp4", granularity: str = "token",
                         rotate: int | None = None, calls: int = 4) -> list[dict[str, Any]]:
    """quant.py:1575-1653: which ``nn.Linear`` layers of ``module`` to keep in FP8 W8A8. ``run()``
    calls the module; each layer's first ``calls`` inputs (their rows together) are recorded,
    and the layer is quantised alone to W4A4 (:func:`fp4_w4a4_error`) and to FP8 W8A8
    (:func:`fp8_w8a8_error`) on them. One row per layer, most sensitive first (largest W4A4
    output relative L2): ``name``, ``rows``, ``in_features``, ``out_features``,
    ``activation_crest``, ``w4a4_rel_l2``, ``w4a4_norm_change``, ``fp8_rel_l2``, ``input_group``
    (the first layer that read the same inputs) and ``flop_share`` (of the layers' GEMM
    FLOPs). The quantised products run on this library's tcgen05 GEMMs."""
    with _InputRecorder(module, calls) as recorder, torch.no_grad():
        run()
    inputs = recorder.rows()
    groups = _input_groups(inputs)
    table = []
    for name, x in inputs.items():
        found = _sensitivity_of(recorder.layers[name], x, fmt, granularity, rotate)
        if found is not None:
            table.append({"name": name, **found, "input_group": groups[name]})
    total = sum(row["_flops"] for row in table) or 1
    for row in table:
        row["flop_share"] = _sig(row.pop("_flops") / total)
    table.sort(key=lambda row: row["w4a4_rel_l2"], reverse=True)
    return table
