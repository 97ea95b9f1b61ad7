"""CPU restatement of the reference toolkit's quantisers and linears (test infrastructure).

Reference: ``src/kernel_agent/kernels/quant.py`` (kernel-agent 0.1.0); every function cites
the lines it follows. Arithmetic is fp32, one operation at a time in the reference's order;
GEMM accumulations, which the reference runs through cuBLASLt (bits device-dependent) or a
CPU fp32 matmul, are computed here in float64 and rounded once to fp32.
"""

from __future__ import annotations

import math

import numpy as np

from .formats import (
    F32,
    e2m1_codes,
    e2m1_to_f32,
    e4m3_from_f32,
    e4m3_to_f32,
    e8m0_to_f32,
    f32,
    f32_to_bf16,
    frexp32,
    pack_e2m1,
    round_bf16,
    unpack_e2m1,
)

FP8_MAX = 448.0  # quant.py:98
INT8_MAX = 127.0  # quant.py:760
INT8_STEP = F32(1.0 / 127.0)  # quant.py:764
MX_BLOCK = 32  # quant.py:464
MX_SATURATION_SLACK = 2.0**-10  # quant.py:474
FP4_MAX = 6.0  # quant.py:190
NVFP4_OUTER_STEP = F32(1.0 / (FP4_MAX * 448.0))  # quant.py:1033
FP4_BLOCKS = {"nvfp4": 16, "mxfp4": 32}  # quant.py:194-197
NVFP4_ROUNDING_RATIO = FP4_MAX * (1 + 2.0**-4)  # quant.py:1291
FP4_SATURATION_SLACK = 2.0**-10  # quant.py:1294
E4M3_MIN_NORMAL = 2.0**-6  # quant.py:1296

_ERRSTATE = {"over": "ignore", "invalid": "ignore", "divide": "ignore", "under": "ignore"}


def _rows(x) -> np.ndarray:
    x = f32(x)
    return x.reshape(-1, x.shape[-1])


def _amax_rows(a: np.ndarray) -> np.ndarray:
    """``a.abs().amax(dim=1)``: NaN propagates, an empty row gives 0."""
    if a.shape[1] == 0:
        return np.zeros(a.shape[0], F32)
    return np.abs(a).max(axis=1).astype(F32)


def to_dtype(y: np.ndarray, dtype: str) -> np.ndarray:
    """``y.to(dtype)``: bf16 bit patterns for "bf16", the fp32 values for "f32"."""
    return f32_to_bf16(y) if dtype == "bf16" else f32(y)


# ------------------------------------------------------------------ INT8


def row_scales_int8(a: np.ndarray) -> np.ndarray:
    """quant.py:777-780 ``_row_scales``: ``amax * INT8_STEP`` per row, 1 for a zero row."""
    with np.errstate(**_ERRSTATE):
        amax = _amax_rows(a)
        return np.where(amax > 0, amax * INT8_STEP, F32(1.0)).astype(F32)


def int8_codes(a: np.ndarray, scale: np.ndarray) -> np.ndarray:
    """quant.py:770-774 ``_int8_codes``: ``round(a / scale)`` (IEEE division, nearest even),
    clamped to ±127."""
    with np.errstate(**_ERRSTATE):
        q = np.rint(a / scale[:, None]).astype(F32)
        return np.clip(q, -INT8_MAX, INT8_MAX).astype(np.int8)


def quantize_int8_activations(x, smooth=None) -> tuple[np.ndarray, np.ndarray]:
    """quant.py:823-839: per-token int8 codes and fp32 scales (SmoothQuant ``x / s``)."""
    a = _rows(x)
    if smooth is not None:
        with np.errstate(**_ERRSTATE):
            a = (a / f32(smooth)[None, :]).astype(F32)
    scale = row_scales_int8(a)
    return int8_codes(a, scale), scale


def quantize_int8(weight, smooth=None) -> tuple[np.ndarray, np.ndarray]:
    """quant.py:794-813: per-output-channel int8 weight (``weight * s`` with SmoothQuant)."""
    w = f32(weight)
    if w.ndim != 2:
        raise ValueError(f"expected a 2-D weight [out, in], got shape {tuple(w.shape)}")
    if not np.isfinite(w).all():
        raise ValueError("the weight has non-finite values")
    if smooth is not None:
        w = (w * f32(smooth)[None, :]).astype(F32)
    scale = row_scales_int8(w)
    return int8_codes(w, scale), scale


def int8_matmul(a, b) -> np.ndarray:
    """quant.py:854-885: exact int32 ``a @ bᵀ`` of int8 ``a [M, K]``, ``b [N, K]``."""
    return (np.asarray(a, np.int64) @ np.asarray(b, np.int64).T).astype(np.int32)


def int8_epilogue(acc, xs, sw, bias=None) -> np.ndarray:
    """quant.py:920-922: ``acc.float() * xs[:, None] * sw[None, :] (+ bias.float())`` in fp32,
    left to right (three roundings with a bias)."""
    y = (np.asarray(acc, np.int32).astype(F32) * f32(xs)[:, None]).astype(F32)
    y = (y * f32(sw)[None, :]).astype(F32)
    if bias is not None:
        y = (y + f32(bias)[None, :]).astype(F32)
    return y


def int8_w8a8_linear(x, q, scale, bias=None, smooth=None, out_dtype="bf16") -> np.ndarray:
    """quant.py:901-923: per-token int8 activations, exact int32 products, fp32 epilogue,
    one rounding to the output dtype. Returns ``[rows, N]``."""
    xq, xs = quantize_int8_activations(x, smooth)
    acc = int8_matmul(xq, q)
    return to_dtype(int8_epilogue(acc, xs, scale, bias), out_dtype)


# ------------------------------------------------------------------ FP8 per token / channel


def quantize_fp8_rows(a: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """quant.py:116-118 / 374-376: ``scale = amax / 448`` (IEEE division; 1 for a zero row),
    codes ``(a / scale).clamp(±448)`` to e4m3 (nearest even)."""
    with np.errstate(**_ERRSTATE):
        amax = _amax_rows(a)
        scale = np.where(amax > 0, (amax / F32(FP8_MAX)).astype(F32), F32(1.0)).astype(F32)
        v = np.clip((a / scale[:, None]).astype(F32), -FP8_MAX, FP8_MAX)
        return e4m3_from_f32(v), scale


def quantize_fp8_activations(x) -> tuple[np.ndarray, np.ndarray]:
    """quant.py:361-377: per-token e4m3 codes (bytes) and fp32 scales."""
    return quantize_fp8_rows(_rows(x))


def quantize_fp8(weight) -> tuple[np.ndarray, np.ndarray]:
    """quant.py:101-119: per-output-channel e4m3 weight (refuses non-finite values)."""
    w = f32(weight)
    if w.ndim != 2:
        raise ValueError(f"expected a 2-D weight [out, in], got shape {tuple(w.shape)}")
    if not np.isfinite(w).all():
        raise ValueError("the weight has non-finite values")
    return quantize_fp8_rows(w)


def fp8_w8a8_linear(x, q, scale, bias=None, out_dtype="bf16") -> np.ndarray:
    """quant.py:390-417 (the fp32 path): ``(xq * xs) @ (q * sw)ᵀ (+ bias)``; products of the
    dequantised operands accumulated in float64, rounded to fp32 once."""
    xq, xs = quantize_fp8_activations(x)
    a = (e4m3_to_f32(xq) * f32(xs)[:, None]).astype(F32)
    w = (e4m3_to_f32(q) * f32(scale)[:, None]).astype(F32)
    y = (a.astype(np.float64) @ w.astype(np.float64).T).astype(F32)
    if bias is not None:
        y = (y + f32(bias)[None, :]).astype(F32)
    return to_dtype(y, out_dtype)


# ------------------------------------------------------------------ MXFP8


def mx_scale_exponents(amax, rule: str = "ceil") -> np.ndarray:
    """quant.py:479-495: unbiased power-of-two exponents of block maxima (int32, -127 for a
    zero block, clamped to [-127, 127]). ``ceil``: frexp of ``amax / 448`` (fp32 division),
    minus one at an exact power of two, plus one when ``amax > 448 * 2^e`` in fp32."""
    if rule not in ("ceil", "floor"):
        raise ValueError(f"unknown MXFP8 scale rule {rule!r} (one of ceil, floor)")
    a = f32(amax)
    with np.errstate(**_ERRSTATE):
        if rule == "floor":
            _, ex = frexp32(a)
            e = ex.astype(np.int64) - 1 - 8
        else:
            m, ex = frexp32((a / F32(FP8_MAX)).astype(F32))
            e = ex.astype(np.int64) - (m == F32(0.5))
            p2 = np.exp2(e.astype(np.float64)).astype(F32)
            e = e + (a > (F32(FP8_MAX) * p2).astype(F32))
        e = np.where(a > 0, e, -127)
    return np.clip(e, -127, 127).astype(np.int32)


def quantize_mxfp8(x, rule: str = "ceil") -> tuple[np.ndarray, np.ndarray]:
    """quant.py:506-526: e4m3 codes ``[rows, K]`` and e8m0 scale bytes ``[rows, K / 32]``
    (unswizzled), codes ``(x / 2^e).clamp(±448)`` to e4m3."""
    a = _rows(x)
    rows, k = a.shape
    if k % MX_BLOCK:
        raise ValueError(f"the last dimension {k} is not a multiple of the MXFP8 block (32)")
    blocks = a.reshape(rows, k // MX_BLOCK, MX_BLOCK)
    with np.errstate(**_ERRSTATE):
        bmax = np.abs(blocks).max(axis=-1) if k else np.zeros((rows, 0), F32)
        e = mx_scale_exponents(bmax, rule)
        scales = (e + 127).astype(np.uint8)
        step = e8m0_to_f32(scales)
        v = np.clip((blocks / step[..., None]).astype(F32), -FP8_MAX, FP8_MAX)
    return e4m3_from_f32(v).reshape(rows, k), scales


def dequantize_mxfp8(codes, scales) -> np.ndarray:
    """quant.py:529-537: ``codes * 2^e`` per block of 32, fp32 (exact)."""
    c = e4m3_to_f32(codes)
    rows, k = c.shape
    step = e8m0_to_f32(scales).reshape(rows, k // MX_BLOCK, 1)
    return (c.reshape(rows, k // MX_BLOCK, MX_BLOCK) * step).reshape(rows, k).astype(F32)


def mx_scale_offset(row, col, cols: int):
    """quant.py:540-547: byte offset of scale ``[row, col]`` in the 128 x 4 blocked layout."""
    blocks_per_row = -(-cols // 4)
    block = (row // 128) * blocks_per_row + col // 4
    return block * 512 + (row % 32) * 16 + ((row % 128) // 32) * 4 + col % 4


def swizzle_scales(scales) -> np.ndarray:
    """quant.py:550-564 / 1176-1182: ``[rows, cols]`` scale bytes -> the flat 128 x 4 blocked
    layout (rows padded to 128, columns to 4, padding 0)."""
    s = np.asarray(scales, dtype=np.uint8)
    rows, cols = s.shape
    nrb, ncb = -(-rows // 128), -(-cols // 4)
    out = np.zeros(nrb * 128 * ncb * 4, dtype=np.uint8)
    r, c = np.meshgrid(np.arange(rows), np.arange(cols), indexing="ij")
    out[mx_scale_offset(r, c, cols)] = s
    return out


def unswizzle_scales(flat, rows: int, cols: int) -> np.ndarray:
    """The inverse of :func:`swizzle_scales` on its ``[rows, cols]`` part."""
    r, c = np.meshgrid(np.arange(rows), np.arange(cols), indexing="ij")
    return np.asarray(flat, np.uint8)[mx_scale_offset(r, c, cols)]


def mxfp8_linear(x, q, scales, bias=None, rule="ceil", out_dtype="bf16") -> np.ndarray:
    """quant.py:581-620 (the fp32 path): both operands dequantised (exact), products
    accumulated in float64, rounded to fp32, ``+ bias``."""
    xq, xs = quantize_mxfp8(x, rule)
    a = dequantize_mxfp8(xq, xs).astype(np.float64)
    w = dequantize_mxfp8(q, scales).astype(np.float64)
    y = (a @ w.T).astype(F32)
    if bias is not None:
        y = (y + f32(bias)[None, :]).astype(F32)
    return to_dtype(y, out_dtype)


def mxfp8_linear_codes(xq, xs, q, scales, bias=None, out_dtype="bf16") -> np.ndarray:
    """The MXFP8 GEMM of already quantised activations (codes + unswizzled e8m0 bytes)."""
    a = dequantize_mxfp8(xq, xs).astype(np.float64)
    w = dequantize_mxfp8(q, scales).astype(np.float64)
    y = (a @ w.T).astype(F32)
    if bias is not None:
        y = (y + f32(bias)[None, :]).astype(F32)
    return to_dtype(y, out_dtype)


def silu_mul(gate, up) -> np.ndarray:
    """``F.silu(gate) * up`` in bf16 (triton_fp8_producers.py:136-147, the rounding points of
    eager): ``g / (1 + exp(-g))`` rounded to bf16, times ``up``, rounded to bf16. ``exp`` is
    evaluated in float64 and rounded to fp32 (a correctly rounded fp32 exp)."""
    g, u = f32(gate), f32(up)
    with np.errstate(**_ERRSTATE):
        e = np.exp(-g.astype(np.float64)).astype(F32)
        a = round_bf16((g / (F32(1.0) + e).astype(F32)).astype(F32))
        return round_bf16((a * u).astype(F32))


def rmsnorm(x, weight, eps: float, dtype: str = "bf16") -> np.ndarray:
    """RMSNorm times weight as eager computes it (triton_fp8_producers.py:120-133,
    triton_fp4_producers.py:261-294): ``x * rsqrt(mean(x^2) + eps)`` in fp32 rounded to x's
    dtype, times the weight, rounded again. The mean is taken in float64 and rounded to fp32,
    rsqrt in float64 then fp32 (the device's order of the sum and its rsqrt may differ in
    the last bit, which moves a bf16 / fp16 result on a small share of elements)."""
    a = _rows(x)
    rnd = round_bf16 if dtype == "bf16" else (lambda v: v.astype(np.float16).astype(F32))
    with np.errstate(**_ERRSTATE):
        sq = (a * a).astype(F32).astype(np.float64)
        var = (sq.mean(axis=1) if a.shape[1] else np.zeros(a.shape[0])).astype(F32)
        r = (1.0 / np.sqrt((var + F32(eps)).astype(F32).astype(np.float64))).astype(F32)
        hn = rnd((a * r[:, None]).astype(F32))
        return rnd((hn * f32(weight).reshape(1, -1)).astype(F32))


def mxfp8_saturation(x, scales) -> dict:
    """quant.py:623-660: how MXFP8 scales fit the block maxima of ``x``."""
    a = _rows(x)
    rows, k = a.shape
    nb = k // MX_BLOCK
    s = np.asarray(scales)
    if k % MX_BLOCK or s.shape != (rows, nb):
        raise ValueError(
            f"expected scales [{rows}, {nb}] (rows of x, K / 32, unswizzled) for x "
            f"{tuple(np.shape(x))}, got {tuple(s.shape)}"
        )
    with np.errstate(**_ERRSTATE):
        amax = np.abs(a.reshape(rows, nb, MX_BLOCK)).max(axis=-1).astype(F32)
        step = e8m0_to_f32(s) if s.dtype == np.uint8 else f32(s)
        m, _ = frexp32(step)
        not_pow2 = int(((m != F32(0.5)) & (step > 0)).sum())
        ratio = np.where(amax > 0, (amax / np.maximum(step, F32(1e-38))).astype(F32), F32(0))
        limit = FP8_MAX * (1 + MX_SATURATION_SLACK)
        saturated = int(((ratio > limit) | ((step <= 0) & (amax > 0))).sum())
        ceil = mx_scale_exponents(amax, "ceil").astype(np.float64)
        coarser = int(((step.astype(np.float64) > np.exp2(ceil)) & (amax > 0)).sum())
    blocks = rows * nb
    return {
        "blocks": blocks,
        "saturated": saturated,
        "share": _sig(saturated / blocks) if blocks else 0.0,
        "worst_ratio": _sig(float(ratio.max())) if blocks else 0.0,
        "coarser": coarser,
        "not_pow2": not_pow2,
    }


# ------------------------------------------------------------------ FP4 (NVFP4 / MXFP4)


def _fp4_codes(blocks: np.ndarray, step: np.ndarray) -> np.ndarray:
    """quant.py:1043-1053: packed e2m1 codes of ``blocks / step`` (IEEE division), clamped to
    ±6; a block whose step is 0 gets codes 0."""
    rows = blocks.shape[0]
    with np.errstate(**_ERRSTATE):
        safe = np.where(step > 0, step, F32(1.0)).astype(F32)
        v = np.where(step[..., None] > 0, (blocks / safe[..., None]).astype(F32), F32(0))
        codes = e2m1_codes(np.clip(v, -FP4_MAX, FP4_MAX).astype(F32))
    return pack_e2m1(codes.reshape(rows, -1))


def quantize_fp4_activations(x, fmt="nvfp4", granularity="token"):
    """quant.py:1056-1107: packed codes ``[rows, K / 2]``, block scale bytes ``[rows, K /
    block]`` (e4m3 for NVFP4, e8m0 for MXFP4) and the fp32 outer scale ``[rows]``."""
    if fmt not in FP4_BLOCKS:
        raise ValueError(f"unknown FP4 format {fmt!r} (one of nvfp4, mxfp4)")
    if granularity not in ("token", "tensor"):
        raise ValueError(f"unknown granularity {granularity!r} (token, tensor)")
    block = FP4_BLOCKS[fmt]
    a = _rows(x)
    rows, k = a.shape
    if k % block:
        raise ValueError(f"the last dimension {k} is not a multiple of the {fmt} block ({block})")
    blocks = a.reshape(rows, k // block, block)
    with np.errstate(**_ERRSTATE):
        bmax = np.abs(blocks).max(axis=-1).astype(F32) if k else np.zeros((rows, 0), F32)
        if fmt == "mxfp4":
            m, ex = frexp32(bmax)
            e = ex.astype(np.int64) - 3 + (m > F32(0.75))
            e = np.clip(np.where(bmax > 0, e, -127), -127, 127)
            scales = (e + 127).astype(np.uint8)
            outer = np.ones(rows, F32)
            step = e8m0_to_f32(scales)
        else:
            amax = _amax_rows(a)
            if granularity == "tensor" and rows:
                amax = np.full(rows, amax.max(), F32)
            outer = np.where(amax > 0, (amax * NVFP4_OUTER_STEP).astype(F32), F32(1.0)).astype(F32)
            ratio = (bmax / (outer * F32(FP4_MAX)).astype(F32)[:, None]).astype(F32)
            scales = e4m3_from_f32(np.minimum(ratio, F32(448.0)))
            step = (e4m3_to_f32(scales) * outer[:, None]).astype(F32)
    return _fp4_codes(blocks, step), scales, outer


def quantize_fp4(weight, fmt="nvfp4", unbiased=False, amax=None):
    """quant.py:217-272: packed codes, block scale bytes and the fp32 tensor scale
    (``float(amax) / (6 * 448)`` in double, rounded to fp32; 1 for MXFP4); ``unbiased``: the
    tensor scale times each output channel's :func:`fp4_bias_correction` (fp32 ``[out]``).
    ``amax``: the whole weight's amax when ``weight`` is a slice of its rows (the tensor scale
    is the whole weight's, quant.py:253-254)."""
    w = f32(weight)
    if w.ndim != 2:
        raise ValueError(f"expected a 2-D weight [out, in], got shape {tuple(w.shape)}")
    if fmt not in FP4_BLOCKS:
        raise ValueError(f"unknown FP4 format {fmt!r} (one of nvfp4, mxfp4)")
    block = FP4_BLOCKS[fmt]
    rows, cols = w.shape
    if cols % block:
        raise ValueError(f"in_features {cols} is not a multiple of the {fmt} block ({block})")
    if not np.isfinite(w).all():
        raise ValueError("the weight has non-finite values")
    blocks = w.reshape(rows, cols // block, block)
    with np.errstate(**_ERRSTATE):
        bmax = np.abs(blocks).max(axis=-1).astype(F32)
        if fmt == "nvfp4":
            if amax is None:
                amax = float(bmax.max()) if bmax.size else 0.0
            amax = float(amax)
            ts = F32(amax / (FP4_MAX * 448.0) if amax > 0 else 1.0)
            div = F32(FP4_MAX * float(ts))
            scales = e4m3_from_f32(np.minimum((bmax / div).astype(F32), F32(448.0)))
            step = (e4m3_to_f32(scales) * ts).astype(F32)
        else:
            m, ex = frexp32((bmax / F32(FP4_MAX)).astype(F32))
            ceil_log2 = ex.astype(np.int64) - (m == F32(0.5))
            e = np.where(bmax > 0, ceil_log2, -127)
            scales = (np.clip(e, -127, 127) + 127).astype(np.uint8)
            ts = F32(1.0)
            step = e8m0_to_f32(scales)
        v = np.where(
            step[..., None] > 0,
            (blocks / np.maximum(step, F32(1e-38))[..., None]).astype(F32),
            F32(0),
        )
        codes = e2m1_codes(np.clip(v, -FP4_MAX, FP4_MAX).astype(F32)).reshape(rows, cols)
    packed = pack_e2m1(codes)
    if unbiased:
        ts = (F32(ts) * fp4_bias_correction(w, packed, scales, ts, fmt)).astype(F32)
    return packed, scales, ts


def fp4_bias_correction(x, codes, scales, outer=None, fmt=None) -> np.ndarray:
    """quant.py:1117-1148: per row ``c = sum x^2 / sum x x^`` in float64 with ``x^ = e2m1 *
    scale * outer``; 1 where ``sum x x^`` is not positive or ``c`` is not finite; fp32."""
    a = _rows(x).astype(np.float64)
    rows, k = a.shape
    s = np.asarray(scales, np.uint8)
    fmt = fmt or ("nvfp4" if s.shape[-1] * 16 == k else "mxfp4")
    xh = fp4_values(codes, s, fmt).astype(np.float64)
    if outer is not None:
        o = np.asarray(outer, np.float64).reshape(-1)
        xh = xh * (o if o.size == rows else np.full(rows, o[0]))[:, None]
    num, den = (a * a).sum(axis=1), (a * xh).sum(axis=1)
    with np.errstate(**_ERRSTATE):
        c = num / np.maximum(den, 1e-300)
    ok = (den > 0) & np.isfinite(c)
    return np.where(ok, c, 1.0).astype(F32)


def hadamard(n: int) -> np.ndarray:
    """quant.py:1150-1159: the orthonormal Sylvester-Hadamard matrix of order ``n``, fp32."""
    if n < 1 or n & (n - 1):
        raise ValueError(f"the Hadamard order must be a power of two, got {n}")
    h = np.ones((1, 1), F32)
    while h.shape[0] < n:
        h = np.block([[h, h], [h, -h]]).astype(F32)
    return (h / F32(math.sqrt(n))).astype(F32)


def hadamard_rotate(x, block: int) -> np.ndarray:
    """quant.py:1162-1173: every ``block`` elements along K times ``hadamard(block)``; each
    output a float64 sum of the fp32 products, rounded to fp32 (torch's fp32 matmul orders its
    sum its own way: parity is within a few fp32 units)."""
    a = f32(x)
    k = a.shape[-1]
    if k % block:
        raise ValueError(f"the last dimension {k} is not a multiple of the rotation ({block})")
    h = hadamard(block).astype(np.float64)
    v = a.reshape(-1, k // block, block).astype(np.float64) @ h
    return v.astype(F32).reshape(a.shape)


def fp4_values(codes, scales, fmt="nvfp4") -> np.ndarray:
    """quant.py:1110-1114: exact fp32 ``e2m1 * block scale`` ``[rows, K]``."""
    c = unpack_e2m1(codes)
    rows, k = c.shape
    s = np.asarray(scales, np.uint8)
    sv = e4m3_to_f32(s) if fmt == "nvfp4" else e8m0_to_f32(s)
    nb = s.shape[1]
    return (e2m1_to_f32(c).reshape(rows, nb, k // nb) * sv[..., None]).reshape(rows, k).astype(F32)


def fp4_epilogue(acc, outer, ts, bias=None) -> np.ndarray:
    """quant.py:1254-1256: ``acc * (outer[:, None] * ts) (+ bias.float())`` in fp32."""
    factor = (f32(outer)[:, None] * f32(ts).reshape(1, -1)).astype(F32)
    y = (f32(acc) * factor).astype(F32)
    if bias is not None:
        y = (y + f32(bias)[None, :]).astype(F32)
    return y


def fp4_w4a4_linear(x, codes, scales, ts, bias=None, fmt="nvfp4", granularity="token",
                    out_dtype="bf16", rotate=None, unbiased=False) -> np.ndarray:
    """quant.py:1201-1257 (the fp32 path): activations rotated (``rotate``) and quantised per
    call, block-scaled products accumulated in float64 and rounded to fp32, the outer scale
    times the activations' bias correction (``unbiased``), then the fp32 epilogue and one
    rounding to the output dtype."""
    xr = hadamard_rotate(x, rotate) if rotate else x
    xq, xs, outer = quantize_fp4_activations(xr, fmt, granularity)
    if unbiased:
        outer = (f32(outer) * fp4_bias_correction(xr, xq, xs, outer, fmt)).astype(F32)
    acc = (fp4_values(xq, xs, fmt).astype(np.float64)
           @ fp4_values(codes, scales, fmt).astype(np.float64).T).astype(F32)
    return to_dtype(fp4_epilogue(acc, outer, ts, bias), out_dtype)


def fp4_scale_check(x, scales, outer=None, fmt=None) -> dict:
    """quant.py:1325-1416: how W4A4 activation block scales (bytes, unswizzled) fit the block
    maxima of ``x`` with the given outer scale."""
    a = _rows(x)
    rows, k = a.shape
    s_bytes = np.asarray(scales, np.uint8)
    fmt = fmt or ("nvfp4" if s_bytes.shape[-1] * 16 == k else "mxfp4")
    block = FP4_BLOCKS[fmt]
    nb = k // block if k % block == 0 else -1
    if nb < 0 or s_bytes.shape != (rows, nb):
        raise ValueError(
            f"expected {fmt} scales [{rows}, {max(nb, 0)}] (rows of x, K / {block}, unswizzled) "
            f"for x {tuple(np.shape(x))}, got {tuple(s_bytes.shape)}"
        )
    s = e4m3_to_f32(s_bytes) if fmt == "nvfp4" else e8m0_to_f32(s_bytes)
    if outer is None:
        o = np.ones(rows, F32)
    else:
        o = f32(outer).reshape(-1)
        o = np.full(rows, o[0], F32) if o.size == 1 else o
    with np.errstate(**_ERRSTATE):
        bmax = np.abs(a.reshape(rows, nb, block)).max(axis=-1).astype(F32)
        o2 = np.broadcast_to(o[:, None], (rows, nb))
        finite = np.isfinite(s) & np.isfinite(o2) & (o2 > 0)
        step = np.where(finite, (s * o2).astype(F32), F32(0))
        live = finite & (bmax > 0)
        ratio = np.where(live & (step > 0), (bmax / np.maximum(step, F32(1e-38))).astype(F32), F32(0))
        zero = live & (step <= 0)
        if fmt == "nvfp4":
            safe = np.where(finite, o2, F32(1.0)).astype(F32)
            r = (bmax / (safe * F32(FP4_MAX)).astype(F32)).astype(F32)
            rn = e4m3_to_f32(e4m3_from_f32(np.minimum(r, F32(448.0))))
            r_low = (r * F32(1 - 2.0**-20)).astype(F32)
            rn_low = e4m3_to_f32(e4m3_from_f32(np.minimum(r_low, F32(448.0))))
            bound = np.full(bmax.shape, F32(NVFP4_ROUNDING_RATIO), F32)
            for ref in (rn, rn_low):
                ref_ratio = (bmax / np.maximum((ref * safe).astype(F32), F32(1e-38))).astype(F32)
                sub = (ref > 0) & (ref < F32(E4M3_MIN_NORMAL))
                bound = np.where(sub, np.maximum(bound, ref_ratio), bound)
            underflow = int((zero & (rn_low > 0)).sum())
            representable = e4m3_to_f32(e4m3_from_f32(s)) == s
            coarser = int((live & (s > rn)).sum())
        else:
            bound = np.full(bmax.shape, F32(FP4_MAX), F32)
            underflow = int(zero.sum())
            m, _ = frexp32(s)
            representable = (m == F32(0.5)) & (s > 0)
            mb, eb = frexp32(bmax)
            ceil = eb.astype(np.int64) - 3 + (mb > F32(0.75))
            coarser = int((live & (s > np.exp2(ceil.astype(np.float64)).astype(F32))).sum())
        saturated = int((live & (ratio > (bound * F32(1 + FP4_SATURATION_SLACK)).astype(F32))).sum())
    blocks = rows * nb
    return {
        "format": fmt,
        "blocks": blocks,
        "saturated": saturated,
        "share": _sig(saturated / blocks) if blocks else 0.0,
        "worst_ratio": _sig(float(ratio.max())) if blocks else 0.0,
        "underflow": underflow,
        "nonfinite": int((~finite).sum()),
        "not_representable": int((finite & ~representable).sum()),
        "coarser": coarser,
    }


def _sig(value: float, digits: int = 4) -> float:
    """quant.py:129-130: ``value`` to ``digits`` significant digits."""
    return float(f"{value:.{digits}g}") if np.isfinite(value) else value
