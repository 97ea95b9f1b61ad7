"""FP8 attention prefill (configuration 5): a new API in the style of the reference's
research emulation ``docs/research-scripts/fp8-sm120/fp8lib.py:184-215`` (``emulated_sdpa``,
``mode="qkpv"``).

Q, K and V are quantised to e4m3 with one scale per (batch, head) over ``[S, D]``
(``_fq_last2``, fp8lib.py:173-176: ``amax / 448``, a zero scale replaced by 1); the tcgen05
kernel computes ``S = Q Kᵀ · scale`` on the codes, the causal mask, an online softmax whose
``P`` enters ``P V`` as ``e4m3(p · 448) / 448`` with the row sum taken before that rounding,
and returns bf16. The softmax uses the running row max where the emulation uses the global
one, so ``P``'s codes can differ; the output is judged against fp32 attention by relative L2
and cosine, as the emulation is.
"""

from __future__ import annotations

import math

import torch

from .. import _native as nat

_E4M3 = torch.float8_e4m3fn


def quantize_fp8_heads(t: torch.Tensor, transpose: bool = False) -> tuple[torch.Tensor, torch.Tensor]:
    """``(codes e4m3 [..., S, D], scales fp32 [...])`` with one scale ``amax / 448`` per leading
    index (fp8lib.py:173-176). ``transpose``: codes as ``[..., D, S]`` (the ``Vᵀ`` operand), a
    view of a ``[..., D, S16]`` buffer whose rows are padded with zero codes to a multiple of 16
    (the row stride the attention kernel's tensor map needs)."""
    if t.dim() < 2:
        raise ValueError(f"expected [..., S, D], got shape {tuple(t.shape)}")
    nat.require_cuda(t)
    x = t.contiguous()
    if x.dtype not in nat.DTYPES:
        x = x.float()
    *lead, s, d = x.shape
    heads = math.prod(lead)
    amax = torch.empty(max(heads, 1), dtype=torch.int32, device=x.device)
    codes = torch.empty(*lead, d, (s + 15) // 16 * 16, dtype=_E4M3, device=x.device) if transpose else \
        torch.empty(*lead, s, d, dtype=_E4M3, device=x.device)
    scales = torch.empty(lead, dtype=torch.float32, device=x.device)
    if heads and s and d:
        nat.call("kab_quant_heads_fp8", x.data_ptr(), nat.dtype_code(x), heads, s, d, int(transpose),
                 amax.data_ptr(), codes.data_ptr(), scales.data_ptr(), nat.stream_of(x))
    return (codes[..., :s] if transpose else codes), scales


def attention_fp8(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, is_causal: bool = False,
                  enable_gqa: bool = False, scale: float | None = None) -> torch.Tensor:
    """FP8 ``softmax(Q Kᵀ · scale) V`` over ``q [B, Hq, S, D]``, ``k`` / ``v [B, Hkv, S, D]``
    (``D`` 128 or 64; ``Hq`` a multiple of ``Hkv`` with ``enable_gqa``; any ``S``), the qkpv
    emulation's arithmetic on the tensor cores; returns ``q.dtype`` (bf16) ``[B, Hq, S, D]``."""
    if q.dim() != 4 or k.dim() != 4 or v.dim() != 4:
        raise ValueError("expected 4-D q, k, v [batch, heads, seq, head_dim]")
    b, hq, s, d = q.shape
    if k.shape != v.shape or k.shape[0] != b or k.shape[2] != s or k.shape[3] != d:
        raise ValueError(f"k {tuple(k.shape)} / v {tuple(v.shape)} do not match q {tuple(q.shape)}")
    hkv = k.shape[1]
    if hkv != hq and not (enable_gqa and hq % hkv == 0):
        raise ValueError(f"{hq} query heads and {hkv} key / value heads need enable_gqa=True and a multiple")
    if d not in (128, 64):
        raise ValueError(f"head_dim {d}: the FP8 attention kernel takes 128 or 64")
    nat.require_cuda(q, k, v)
    qc, qs = quantize_fp8_heads(q)
    kc, ks = quantize_fp8_heads(k)
    vt, vs = quantize_fp8_heads(v, transpose=True)
    out = torch.empty(b, hq, s, d, dtype=torch.bfloat16, device=q.device)
    sm = float(scale) if scale is not None else d ** -0.5
    nat.call("kab_attention_fp8", qc.data_ptr(), qs.data_ptr(), kc.data_ptr(), ks.data_ptr(), vt.data_ptr(),
             vs.data_ptr(), b, hq, hkv, s, d, int(bool(is_causal)), sm, out.data_ptr(), nat.stream_of(q))
    return out if q.dtype == torch.bfloat16 else out.to(q.dtype)


def emulated_sdpa(q, k, v, attn_mask=None, is_causal=False, enable_gqa=False, scale=None, mode="none",
                  kv_scale=None) -> torch.Tensor:
    """fp8lib.py:184-215 with its signature: ``mode="qkpv"`` runs :func:`attention_fp8`; the
    emulation's other modes and explicit masks are not built on the GPU."""
    if mode != "qkpv":
        raise NotImplementedError(f"emulated_sdpa(mode={mode!r}): only 'qkpv' runs on the GPU kernel")
    if attn_mask is not None:
        raise NotImplementedError("emulated_sdpa: explicit attention masks are not built (is_causal is)")
    return attention_fp8(q, k, v, is_causal=is_causal, enable_gqa=enable_gqa, scale=scale)
