"""Number formats of the oracle (test infrastructure only): bf16, e4m3fn, e8m0, e2m1.

Each encoder restates the conversion torch performs on the CPU for the reference
(``c10/util/Float8_e4m3fn.h`` style round-to-nearest-even with the e4m3fn NaN pattern 0x7F,
``c10/util/BFloat16.h`` round-to-nearest-even with the canonical NaN 0x7FC0), and the e2m1
rounding of ``src/kernel_agent/kernels/quant.py:204-214`` (``_round_e2m1``).
"""

from __future__ import annotations

import numpy as np

F32 = np.float32

#: e2m1 magnitudes of codes 0..7 (quant.py:189).
E2M1_VALUES = (0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0)
#: midpoints between e2m1 magnitudes and the ones a tie rounds up at (quant.py:200-201).
E2M1_MIDPOINTS = (0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0)
E2M1_TIE_UP = (0.75, 1.75, 3.5)


def f32(a) -> np.ndarray:
    """``a`` as a float32 array (no copy when it already is one)."""
    return np.asarray(a, dtype=F32)


# ------------------------------------------------------------------ bf16


def bf16_to_f32(bits) -> np.ndarray:
    """fp32 values of bf16 bit patterns (uint16)."""
    u = np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16
    return u.view(F32)


def f32_to_bf16(v) -> np.ndarray:
    """bf16 bit patterns (uint16) of fp32 values, round to nearest even; NaN -> 0x7FC0."""
    v = f32(v)
    b = v.view(np.uint32).astype(np.uint64)
    r = ((b + 0x7FFF + ((b >> 16) & 1)) >> 16).astype(np.uint16)
    return np.where(np.isnan(v), np.uint16(0x7FC0), r).astype(np.uint16)


def round_bf16(v) -> np.ndarray:
    """fp32 values rounded to bf16 and back (one ``.to(torch.bfloat16).float()``)."""
    return bf16_to_f32(f32_to_bf16(v))


# ------------------------------------------------------------------ e4m3fn


def e4m3_from_f32(v) -> np.ndarray:
    """e4m3fn bytes of fp32 values, round to nearest even (the reference clamps to ±448
    first). |v| >= 480, inf and NaN give 0x7F (NaN) with the sign bit, as torch's CPU
    conversion; below 2^-6 steps of 2^-9 (subnormal); the sign of zero is kept."""
    v = f32(v)
    bits = v.view(np.uint32).astype(np.int64)
    sign = ((bits >> 24) & 0x80).astype(np.uint8)
    f = bits & 0x7FFFFFFF
    out = np.zeros(v.shape, dtype=np.int64)
    big = f >= 0x43F00000  # 480: the first value past 448 + half a step, inf, NaN
    den = f < (121 << 23)  # below 2^-6
    nrm = ~big & ~den
    out[den] = np.rint(np.abs(v[den]).astype(np.float64) * 512.0).astype(np.int64)
    fn = f[nrm]
    out[nrm] = (fn + ((7 - 127) << 23) + 0x7FFFF + ((fn >> 20) & 1)) >> 20
    out[big] = 0x7F
    return out.astype(np.uint8) | sign


def e4m3_to_f32(code) -> np.ndarray:
    """fp32 values of e4m3fn bytes (0x7F / 0xFF: NaN)."""
    c = np.asarray(code, dtype=np.uint8).astype(np.int64)
    e = (c >> 3) & 0xF
    m = c & 7
    mag = np.where(e == 0, m * 2.0**-9, (1.0 + m / 8.0) * np.exp2((e - 7).astype(np.float64)))
    mag = np.where((c & 0x7F) == 0x7F, np.nan, mag)
    return np.where(c & 0x80, -mag, mag).astype(F32)


def round_e4m3(v) -> np.ndarray:
    """fp32 values rounded to e4m3fn and back."""
    return e4m3_to_f32(e4m3_from_f32(v))


# ------------------------------------------------------------------ e8m0


def e8m0_to_f32(byte) -> np.ndarray:
    """fp32 values of e8m0 bytes: 2^(byte - 127); 255 is NaN; byte 0 is 2^-127 (an fp32
    subnormal)."""
    b = np.asarray(byte, dtype=np.uint8).astype(np.float64)
    v = np.exp2(b - 127.0)
    return np.where(b == 255, np.nan, v).astype(F32)


# ------------------------------------------------------------------ e2m1


def e2m1_codes(v) -> np.ndarray:
    """e2m1 codes (uint8 0..15, one per element) of fp32 values within ±6: the midpoint
    comparisons of quant.py:204-214 (ties at 0.75 / 1.75 / 3.5 up, at 0.25 / 1.25 / 2.5 / 5
    down), sign in bit 3, no negative zero."""
    v = f32(v)
    mag = np.abs(v)
    idx = np.zeros(v.shape, dtype=np.int64)
    for mid in E2M1_MIDPOINTS:
        idx += (mag >= mid) if mid in E2M1_TIE_UP else (mag > mid)
    negative = (v < 0) & (idx > 0)
    return (idx + 8 * negative).astype(np.uint8)


def e2m1_to_f32(code) -> np.ndarray:
    """fp32 values of e2m1 codes 0..15."""
    lut = np.array(E2M1_VALUES + tuple(-x for x in E2M1_VALUES), dtype=F32)
    return lut[np.asarray(code, dtype=np.uint8) & 0xF]


def pack_e2m1(codes) -> np.ndarray:
    """Two e2m1 codes per byte along the last axis, the even element in the low nibble
    (quant.py:268, 1053)."""
    c = np.asarray(codes, dtype=np.uint8)
    return (c[..., 0::2] | (c[..., 1::2] << 4)).astype(np.uint8)


def unpack_e2m1(packed) -> np.ndarray:
    """The codes of :func:`pack_e2m1`'s bytes, in element order."""
    p = np.asarray(packed, dtype=np.uint8)
    out = np.empty(p.shape[:-1] + (2 * p.shape[-1],), dtype=np.uint8)
    out[..., 0::2] = p & 0xF
    out[..., 1::2] = p >> 4
    return out


# ------------------------------------------------------------------ frexp of fp32


def frexp32(v) -> tuple[np.ndarray, np.ndarray]:
    """``torch.frexp`` of fp32 values: mantissa in [0.5, 1) (fp32) and int32 exponent;
    0 -> (0, 0); subnormals normalised."""
    m, e = np.frexp(f32(v))
    return m.astype(F32), e.astype(np.int32)
