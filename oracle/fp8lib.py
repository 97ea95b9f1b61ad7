"""CPU restatement of the reference's blockwise-FP8 and FP8-attention math (test
infrastructure only).

Reference: ``docs/research-scripts/fp8-sm120/fp8lib.py`` (``q8`` 12-14, ``_safe`` 17-18,
``fq_groups`` 22-27, ``fq_block`` 35-39, ``_fq_last2`` 173-176, ``emulated_sdpa`` 184-215) and
the blockwise GEMM's promotion rule of ``docs/research-scripts/fp8-sm120/gemm_bench.py:39-68``
(``_bw_gemm``: one fp32 partial product per 128-wide K step, multiplied by both scales and
added into the fp32 accumulator). The toolkit has no blockwise or attention function; these
are the formulas the new APIs follow (parity unpinned beyond them: no reference test holds a
known answer for either).
"""

from __future__ import annotations

import numpy as np

from .formats import F32, e4m3_from_f32, e4m3_to_f32, f32, f32_to_bf16

FMAX = 448.0
_ERR = {"over": "ignore", "invalid": "ignore", "divide": "ignore", "under": "ignore"}


def _safe(s: np.ndarray) -> np.ndarray:
    """fp8lib.py:17-18: a scale of 0 becomes 1."""
    return np.where(s > 0, s, F32(1.0)).astype(F32)


def q8_codes(v: np.ndarray) -> np.ndarray:
    """fp8lib.py:12-14 without the way back: ``v.clamp(±448)`` to e4m3 bytes."""
    return e4m3_from_f32(np.clip(f32(v), -FMAX, FMAX))


def quantize_fp8_groups(x, group: int = 128) -> tuple[np.ndarray, np.ndarray]:
    """fp8lib.py:22-27 ``fq_groups``: one scale ``amax / 448`` (``_safe``) per ``1 x group``
    along the last dimension. Returns e4m3 codes ``[R, K]`` and fp32 scales ``[R, K / group]``."""
    a = f32(x).reshape(-1, np.shape(x)[-1])
    r, k = a.shape
    if k % group:
        raise ValueError(f"the last dimension {k} is not a multiple of the group ({group})")
    g = a.reshape(r, k // group, group)
    with np.errstate(**_ERR):
        s = _safe((np.abs(g).max(axis=-1) / F32(FMAX)).astype(F32))
        codes = q8_codes((g / s[..., None]).astype(F32))
    return codes.reshape(r, k), s


def quantize_fp8_blocks(w, block: int = 128) -> tuple[np.ndarray, np.ndarray]:
    """fp8lib.py:35-39 ``fq_block``: one scale per ``block x block`` tile of a 2-D weight.
    Returns e4m3 codes ``[N, K]`` and fp32 scales ``[N / block, K / block]``."""
    a = f32(w)
    n, k = a.shape
    if n % block or k % block:
        raise ValueError(f"weight {tuple(a.shape)} is not a whole number of {block} x {block} blocks")
    g = a.reshape(n // block, block, k // block, block)
    with np.errstate(**_ERR):
        s = _safe((np.abs(g).max(axis=(1, 3)) / F32(FMAX)).astype(F32))
        codes = q8_codes((g / s[:, None, :, None]).astype(F32))
    return codes.reshape(n, k), s


def fp8_blockwise_gemm(xq, xs, wq, ws, bias=None, out_dtype="bf16", group: int = 128) -> np.ndarray:
    """gemm_bench.py:39-68 ``_bw_gemm``: for each 128-wide K step a partial product of the
    e4m3 codes (exact in float64, rounded to fp32), then ``acc += part * sa[m, kb] * sb[nb,
    kb]`` as the Triton kernel compiles it (default fp fusion: ``t = part * sa`` rounded to
    fp32, then ``acc = fma(t, sb, acc)``); ``+ bias``; one rounding to the output dtype.

    The fused multiply-add is taken in float64 (``t * sb`` is exact there, 48 significant
    bits) and rounded to fp32; that double rounding can differ from a single one by one fp32
    unit in the last place in rare ties, far below the tests' bf16 tolerance."""
    a = e4m3_to_f32(xq).astype(np.float64)
    b = e4m3_to_f32(wq).astype(np.float64)
    m, k = a.shape
    n = b.shape[0]
    nkb = k // group
    acc = np.zeros((m, n), F32)
    sb_full = np.repeat(f32(ws), group, axis=0)[:n]  # [N, nkb]
    for kb in range(nkb):
        sl = slice(kb * group, (kb + 1) * group)
        part = (a[:, sl] @ b[:, sl].T).astype(F32)
        t = (part * f32(xs)[:, kb : kb + 1]).astype(F32)
        acc = (t.astype(np.float64) * sb_full[None, :, kb].astype(np.float64) + acc.astype(np.float64)).astype(F32)
    if bias is not None:
        acc = (acc + f32(bias)[None, :]).astype(F32)
    return f32_to_bf16(acc) if out_dtype == "bf16" else acc


def quantize_head(t) -> tuple[np.ndarray, np.ndarray]:
    """fp8lib.py:173-176 ``_fq_last2``: one scale ``amax / 448`` (``_safe``) per leading index
    over the last two dimensions ``[S, D]``. Returns e4m3 codes and fp32 scales ``t.shape[:-2]``."""
    a = f32(t)
    with np.errstate(**_ERR):
        s = _safe((np.abs(a).max(axis=(-2, -1)) / F32(FMAX)).astype(F32))
        codes = q8_codes((a / s[..., None, None]).astype(F32))
    return codes, s


def attention_fp8_head(q, k, v, causal: bool = True, scale: float | None = None) -> np.ndarray:
    """fp8lib.py:184-215 ``emulated_sdpa(mode="qkpv")`` for one (batch, head): Q, K, V
    fake-quantised per head (one e4m3 scale over ``[S, D]``), ``s = q kᵀ * scale`` (float64
    products), causal mask, ``p = exp(s - rowmax)``, ``denom = Σ p`` before P is rounded,
    P as ``e4m3(p * 448) / 448``, ``out = (P v) / denom``. Returns fp32 ``[Sq, D]``."""
    qc, qs = quantize_head(q)
    kc, ks = quantize_head(k)
    vc, vs = quantize_head(v)
    qf = (e4m3_to_f32(qc) * qs).astype(np.float64)
    kf = (e4m3_to_f32(kc) * ks).astype(np.float64)
    vf = (e4m3_to_f32(vc) * vs).astype(np.float64)
    d = qf.shape[-1]
    sc = float(scale) if scale is not None else d**-0.5
    s = (qf @ kf.T) * sc
    if causal:
        lq, lk = s.shape
        s = np.where(np.triu(np.ones((lq, lk), bool), 1), -np.inf, s)
    m = s.max(axis=-1, keepdims=True)
    p = np.exp(s - m)
    denom = p.sum(axis=-1, keepdims=True)
    p8 = e4m3_to_f32(q8_codes((p * FMAX).astype(F32))).astype(np.float64) / FMAX
    return ((p8 @ vf) / denom).astype(F32)


def attention_fp8(q, k, v, causal: bool = True, heads=None) -> np.ndarray:
    """``emulated_sdpa(q, k, v, is_causal, enable_gqa=True, mode="qkpv")`` over ``[B, Hq, S,
    D]`` / ``[B, Hkv, S, D]``, head by head (``heads``: an optional list of ``(b, h)`` pairs to
    compute, the rest left 0). Returns fp32 ``[B, Hq, S, D]``."""
    q, k, v = f32(q), f32(k), f32(v)
    b_, hq, sq, d = q.shape
    rep = hq // k.shape[1]
    out = np.zeros(q.shape, F32)
    for b in range(b_):
        for h in range(hq):
            if heads is not None and (b, h) not in heads:
                continue
            out[b, h] = attention_fp8_head(q[b, h], k[b, h // rep], v[b, h // rep], causal)
    return out


def sdpa_fp32(q, k, v, causal: bool = True) -> np.ndarray:
    """Plain attention in float64 (the unquantised reference the FP8 output is judged
    against), GQA by head index, fp32 result."""
    q, k, v = (np.asarray(t, np.float64) for t in (q, k, v))
    b_, hq, sq, d = q.shape
    rep = hq // k.shape[1]
    out = np.zeros(q.shape, F32)
    for b in range(b_):
        for h in range(hq):
            s = q[b, h] @ k[b, h // rep].T * d**-0.5
            if causal:
                s = np.where(np.triu(np.ones(s.shape, bool), 1), -np.inf, s)
            p = np.exp(s - s.max(axis=-1, keepdims=True))
            out[b, h] = ((p @ v[b, h // rep]) / p.sum(axis=-1, keepdims=True)).astype(F32)
    return out
