"""CPU restatement of the reference's FP8 KV-cache math (test infrastructure only).

Reference: ``src/kernel_agent/kernels/kv_quant.py`` (kernel-agent 0.1.0): ``quantize_fp8_kv``
38-46, ``dequantize_fp8_kv`` 49-53, ``fp8_kv_attention`` 56-83, ``fp8_kv_error`` 86-101,
``Fp8KVCache.append`` 133-151 and ``kv_cache_share`` 160-183. The quantiser's arithmetic is
fp32, one operation at a time in the reference's order (pinned bit for bit by
``tests/golden/kv_golden.npz``); the attention is computed in float64 and rounded once to
fp32 (the reference's fp32 matmuls round in a device-dependent order).
"""

from __future__ import annotations

import math

import numpy as np

from .formats import F32, e4m3_from_f32, e4m3_to_f32, f32

E4M3_MAX = 448.0  # kv_quant.py:35

_ERR = {"over": "ignore", "invalid": "ignore", "divide": "ignore", "under": "ignore"}


def quantize_fp8_kv(t) -> tuple[np.ndarray, np.ndarray]:
    """kv_quant.py:38-46: ``(codes, scales)`` of ``t [..., tokens, D]``: e4m3 bytes of ``t``'s
    shape and fp32 scales ``[..., tokens]``: ``amax(|row|) / 448`` where ``amax > 0`` (the
    quotient, even when it underflows to 0), else 1 (zero rows and NaN); codes
    ``clamp(t / scale, ±448)`` rounded to nearest even."""
    a = f32(t)
    with np.errstate(**_ERR):
        amax = (np.abs(a).max(axis=-1) if a.shape[-1] else np.zeros(a.shape[:-1])).astype(F32)
        scale = np.where(amax > 0, (amax / F32(E4M3_MAX)).astype(F32), F32(1.0)).astype(F32)
        q = (a / scale[..., None]).astype(F32)
        codes = e4m3_from_f32(np.clip(q, -E4M3_MAX, E4M3_MAX))
    return codes, scale


def dequantize_fp8_kv(codes, scales) -> np.ndarray:
    """kv_quant.py:49-53: ``codes * scales[..., None]`` in fp32."""
    with np.errstate(**_ERR):
        return (e4m3_to_f32(codes) * f32(scales)[..., None]).astype(F32)


def fp8_kv_attention(q, k_codes, k_scales, v_codes, v_scales, scale=None, lengths=None) -> np.ndarray:
    """kv_quant.py:56-83: ``softmax(Q Kᵀ · scale) V`` over the dequantised cache. ``q
    [B, Hq, Lq, D]`` (fp32 values), codes ``[B, Hkv, L, D]``, scales ``[B, Hkv, L]``;
    grouped-query heads by repetition; ``lengths [B]``: the valid cached tokens per
    sequence. Returns fp32 ``[B, Hq, Lq, D]``."""
    qf = np.asarray(q, np.float64)
    k = dequantize_fp8_kv(k_codes, k_scales).astype(np.float64)
    v = dequantize_fp8_kv(v_codes, v_scales).astype(np.float64)
    rep = qf.shape[1] // k.shape[1]
    if rep > 1:
        k, v = np.repeat(k, rep, axis=1), np.repeat(v, rep, axis=1)
    sm = qf.shape[-1] ** -0.5 if scale is None else float(scale)
    with np.errstate(**_ERR):
        s = np.einsum("bhqd,bhkd->bhqk", qf, k) * sm
        if lengths is not None:
            valid = np.arange(k.shape[2])[None, :] < np.asarray(lengths)[:, None]
            s = np.where(valid[:, None, None, :], s, -np.inf)
        m = s.max(axis=-1, keepdims=True)
        p = np.exp(s - m)
        out = np.einsum("bhqk,bhkd->bhqd", p / p.sum(axis=-1, keepdims=True), v)
    return out.astype(F32)


def fp8_kv_error(k, v) -> dict:
    """kv_quant.py:86-101: relative L2 error of K and V after the e4m3 round trip, the worst
    per-(token, head) row, and the bytes before / after (``element_bytes`` of the input)."""
    report: dict = {"format": "float8_e4m3fn", "granularity": "per token and head"}
    for name, t in (("k", k), ("v", v)):
        a = f32(t).astype(np.float64)
        deq = dequantize_fp8_kv(*quantize_fp8_kv(f32(t))).astype(np.float64)
        norm = float(np.linalg.norm(a))
        rows = np.linalg.norm(deq - a, axis=-1) / np.maximum(np.linalg.norm(a, axis=-1), 1e-30)
        report[f"{name}_rel_l2"] = round(float(np.linalg.norm(deq - a)) / norm, 5) if norm else 0.0
        report[f"{name}_worst_row_rel_l2"] = round(float(rows.max()), 5) if rows.size else 0.0
    return report


def fp8_kv_bytes(k_shape, element_bytes: int) -> dict:
    """kv_quant.py:98-100: bytes before (K and V in their dtype) and after (codes + one fp32
    scale per token and head)."""
    elems = 2 * math.prod(k_shape)
    rows = elems // max(k_shape[-1], 1)
    return {"before": elems * element_bytes, "after": elems + 4 * rows}


def kv_cache_share(*, batch, tokens, layers, kv_heads, head_dim, other_bytes, elem_bytes=2.0) -> dict:
    """kv_quant.py:160-183: the KV cache's bytes per decode step, its share of the step's
    bytes and the share e4m3 K / V (one fp32 scale per token and head) would save."""
    rows = 2 * batch * tokens * layers * kv_heads
    kv = rows * head_dim * elem_bytes
    fp8 = rows * (head_dim + 4)
    total = kv + other_bytes
    return {
        "kv_bytes": kv,
        "share": kv / total if total else 0.0,
        "saved_share": max(kv - fp8, 0.0) / total if total else 0.0,
    }
