"""FP8 KV cache on the GPU: the drop-in of ``kernel_agent.kernels.kv_quant`` and of the decode
example ``src/kernel_agent/agent/examples/triton_fp8_kv_decode.py``.

K and V get one fp32 scale per (token, KV head), ``amax / 448`` over the head dimension,
written once when tokens are appended (kv_quant.py:1-13). The decode attention reads the
codes and scales directly: the CUDA kernel (``kab_kv_decode_fp8``) feeds the e4m3 K and V
tiles to the tcgen05 tensor cores as they are, with the bf16 query and the softmax weights
carried as exact two-term e4m3 splits; splits of the cache run in parallel and are merged in
the same launch.

* :func:`quantize_fp8_kv` / :func:`dequantize_fp8_kv` (kv_quant.py:38-53), and
  :func:`quantize_kv`, the example's name for the same quantiser.
* :func:`fp8_kv_attention` (kv_quant.py:56-83) and :func:`fp8_kv_decode`
  (triton_fp8_kv_decode.py:195-260): softmax(Q Kᵀ · scale) V over the cache, grouped-query
  heads, optional per-sequence lengths.
* :class:`Fp8KVCache` (kv_quant.py:104-151): a preallocated e4m3 cache whose ``append``
  quantises the new tokens straight into their slots.
* :func:`fp8_kv_error` and :func:`kv_cache_share` (kv_quant.py:86-101, 154-183).
* :class:`Fp8KVDecodeAttention` / :func:`build` (triton_fp8_kv_decode.py:279-300).
"""

from __future__ import annotations

import ctypes
import math
from typing import Any

import torch
from torch import nn

from .. import _native as nat

#: Largest finite e4m3 value (kv_quant.py:35).
E4M3_MAX = 448.0
_E4M3 = torch.float8_e4m3fn
_HEAD_DIMS = (16, 32, 64, 128, 256)


def _check_head_dim(d: int) -> None:
    if d not in _HEAD_DIMS:
        raise ValueError(f"head_dim {d}: the FP8 KV quantiser takes a power of two in 16..256")


def _kv_input(t: torch.Tensor) -> torch.Tensor:
    x = t.detach()
    if x.dtype not in nat.DTYPES:
        x = x.float()
    return x.contiguous()


def quantize_fp8_kv(t: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """``(codes, scales)`` of K or V ``t [..., tokens, head_dim]`` (kv_quant.py:38-46): e4m3
    codes of ``t``'s shape and fp32 scales ``[..., tokens]``, one per (token, head):
    ``amax(|row|) / 448`` (1 for a row of zeros), codes ``round(t / scale)`` to nearest even,
    clamped to ±448. Bit-identical to the reference."""
    if t.dim() < 1:
        raise ValueError("expected [..., head_dim]")
    d = t.shape[-1]
    _check_head_dim(d)
    nat.require_cuda(t)
    x = _kv_input(t)
    codes = torch.empty(x.shape, dtype=_E4M3, device=x.device)
    scales = torch.empty(x.shape[:-1], dtype=torch.float32, device=x.device)
    rows = x.numel() // d
    if rows:
        nat.call("kab_quant_kv_fp8", x.data_ptr(), nat.dtype_code(x), rows, 1, d, d, 0, codes.data_ptr(), d, 0,
                 scales.data_ptr(), 1, 0, nat.stream_of(x))
    return codes, scales


#: The example's name for the GPU quantiser (triton_fp8_kv_decode.py:176-190).
quantize_kv = quantize_fp8_kv


def dequantize_fp8_kv(codes: torch.Tensor, scales: torch.Tensor, dtype: torch.dtype = torch.float32) -> torch.Tensor:
    """The values of :func:`quantize_fp8_kv`'s ``(codes, scales)`` in ``dtype``
    (kv_quant.py:49-53: the product in fp32, one rounding to ``dtype``)."""
    nat.require_cuda(codes, scales)
    return (codes.float() * scales.float()[..., None]).to(dtype)


# ------------------------------------------------------------------ decode attention

_WORKSPACES: dict[tuple[int, int], torch.Tensor] = {}
_PARAMS: dict[tuple, tuple[bytes, int]] = {}


def _workspace(device: torch.device, stream: int, nbytes: int) -> torch.Tensor:
    """A zeroed scratch buffer per (device, stream): the kernel leaves its split counters at
    zero, so the buffer is zeroed only when it is (re)allocated, on the stream that uses it."""
    key = (device.index if device.index is not None else torch.cuda.current_device(), stream)
    buf = _WORKSPACES.get(key)
    if buf is None or buf.numel() < nbytes:
        buf = torch.zeros(max(nbytes, 1 << 16), dtype=torch.uint8, device=device)
        _WORKSPACES[key] = buf
    return buf


def _unit_last(t: torch.Tensor) -> torch.Tensor:
    return t if t.stride(-1) == 1 else t.contiguous()


def _decode(q4: torch.Tensor, k_codes, k_scales, v_codes, v_scales, scale, lengths, splits) -> torch.Tensor:
    """The kernel over ``q4 [B, Hq, Lq, D]``: every query token sees every valid token."""
    if k_codes.dim() != 4 or v_codes.shape != k_codes.shape:
        raise ValueError(f"codes must be [batch, kv_heads, tokens, head_dim]; got K {tuple(k_codes.shape)}, "
                         f"V {tuple(v_codes.shape)}")
    b, hkv, length, d = k_codes.shape
    if q4.shape[0] != b or q4.shape[3] != d or q4.shape[1] % hkv:
        raise ValueError(f"q {tuple(q4.shape)} does not fit the cache {tuple(k_codes.shape)}")
    if k_scales.shape != (b, hkv, length) or v_scales.shape != (b, hkv, length):
        raise ValueError(f"scales must be [batch, kv_heads, tokens] = {(b, hkv, length)}")
    if k_codes.dtype != _E4M3 or v_codes.dtype != _E4M3:
        raise ValueError("the codes must be float8_e4m3fn")
    if length < 1:
        raise ValueError("an empty cache: at least one token is needed")
    nat.require_cuda(q4, k_codes, k_scales, v_codes, v_scales)
    hq, lq = q4.shape[1], q4.shape[2]
    if d not in (64, 128):
        raise NotImplementedError(f"head_dim {d}: the FP8 KV decode kernel takes 64 or 128")
    if hq // hkv * lq > 32:
        raise NotImplementedError(f"{hq // hkv} query heads per KV head x {lq} query tokens: the kernel takes "
                                  "at most 32 rows per KV head")
    qx = q4 if q4.dtype in nat.DTYPES else q4.float()
    # rows of one KV head's group (query heads x query tokens) at one stride
    if qx.stride(-1) != 1 or (lq > 1 and qx.stride(1) != lq * qx.stride(2)):
        qx = qx.contiguous()
    row_stride = qx.stride(2) if lq > 1 else qx.stride(1)
    k_codes, v_codes = _unit_last(k_codes), _unit_last(v_codes)
    k_scales = _unit_last(k_scales.float() if k_scales.dtype != torch.float32 else k_scales)
    v_scales = _unit_last(v_scales.float() if v_scales.dtype != torch.float32 else v_scales)
    lens = None
    if lengths is not None:
        lens = torch.as_tensor(lengths, device=qx.device).to(torch.int32).contiguous()
        if lens.shape != (b,):
            raise ValueError(f"lengths must be [batch] = [{b}]")
    out = torch.empty(b, hq, lq, d, dtype=torch.bfloat16, device=qx.device)
    stream = nat.stream_of(qx)
    key = (qx.device.index, qx.dtype, tuple(qx.shape), qx.stride(0), row_stride, tuple(k_codes.shape),
           k_codes.stride(), v_codes.stride(), k_scales.stride()[:2], v_scales.stride()[:2], lens is None,
           scale, int(splits))
    cached = _PARAMS.get(key)
    if cached is None:  # the launch's fixed fields and workspace size, once per shape
        t = nat.KabKvDecodeParams()
        t.q_dtype, t.q_stride_b, t.q_stride_row = nat.dtype_code(qx), qx.stride(0), row_stride
        t.kc_stride_b, t.kc_stride_h, t.kc_stride_l = k_codes.stride()[:3]
        t.vc_stride_b, t.vc_stride_h, t.vc_stride_l = v_codes.stride()[:3]
        t.ks_stride_b, t.ks_stride_h = k_scales.stride()[:2]
        t.vs_stride_b, t.vs_stride_h = v_scales.stride()[:2]
        t.batch, t.heads_q, t.heads_kv, t.q_len, t.length, t.head_dim = b, hq, hkv, lq, length, d
        t.sm_scale = float(d ** -0.5 if scale is None else scale)
        t.splits = int(splits)
        nsplit, nbytes = ctypes.c_int(0), ctypes.c_size_t(0)
        nat.call("kab_kv_decode_workspace", ctypes.byref(t), ctypes.byref(nsplit), ctypes.byref(nbytes))
        cached = _PARAMS[key] = (bytes(t), int(nbytes.value))
    template, nbytes = cached
    p = nat.KabKvDecodeParams.from_buffer_copy(template)
    p.q, p.k_codes, p.k_scales = qx.data_ptr(), k_codes.data_ptr(), k_scales.data_ptr()
    p.v_codes, p.v_scales, p.out = v_codes.data_ptr(), v_scales.data_ptr(), out.data_ptr()
    p.lengths = None if lens is None else lens.data_ptr()
    ws = _workspace(qx.device, stream, nbytes) if nbytes else None
    nat.call("kab_kv_decode_fp8", ctypes.byref(p), None if ws is None else ws.data_ptr(),
             0 if ws is None else ws.numel(), stream)
    return out


def fp8_kv_decode(q: torch.Tensor, k_codes: torch.Tensor, k_scales: torch.Tensor, v_codes: torch.Tensor,
                  v_scales: torch.Tensor, scale: float | None = None, lengths: torch.Tensor | None = None,
                  splits: int = 0) -> torch.Tensor:
    """Decode attention of one query token per sequence over an e4m3 cache
    (triton_fp8_kv_decode.py:195-260): q ``[B, Hq, D]`` or ``[B, Hq, 1, D]``, codes
    ``[B, Hkv, L, D]``, scales ``[B, Hkv, L]`` (any strides with a unit last stride),
    ``lengths [B]`` (valid tokens per sequence, >= 1). Returns ``q``'s shape in bf16.
    ``splits``: chunks of the cache per (sequence, KV head), 0 for one wave of CTAs."""
    if q.dim() == 3:
        q4 = q.unsqueeze(2)
    elif q.dim() == 4 and q.shape[2] == 1:
        q4 = q
    else:
        raise ValueError(f"q must be [B, Hq, D] or [B, Hq, 1, D]; got {tuple(q.shape)}")
    return _decode(q4, k_codes, k_scales, v_codes, v_scales, scale, lengths, splits).reshape(q.shape)


def fp8_kv_attention(q: torch.Tensor, k_codes: torch.Tensor, k_scales: torch.Tensor, v_codes: torch.Tensor,
                     v_scales: torch.Tensor, scale: float | None = None,
                     lengths: torch.Tensor | None = None) -> torch.Tensor:
    """softmax(Q Kᵀ · scale) V over an e4m3 cache (kv_quant.py:56-83), returned in ``q``'s
    dtype: ``q [B, Hq, Lq, D]``, codes ``[B, Hkv, L, D]`` and scales ``[B, Hkv, L]`` (Hq a
    multiple of Hkv), ``scale`` default ``D ** -0.5``, ``lengths [B]`` the valid cached
    tokens per sequence. Every query sees every valid cached token. Runs the decode kernel
    (up to 32 query rows per KV head, head_dim 64 or 128); the output is bf16-rounded."""
    if q.dim() != 4:
        raise ValueError(f"q must be [B, Hq, Lq, D]; got {tuple(q.shape)}")
    out = _decode(q, k_codes, k_scales, v_codes, v_scales, scale, lengths, 0)
    return out if q.dtype == torch.bfloat16 else out.to(q.dtype)


# ------------------------------------------------------------------ reports and the cache


def fp8_kv_error(k: torch.Tensor, v: torch.Tensor) -> dict[str, Any]:
    """Error report of an e4m3 cache (kv_quant.py:86-101): relative L2 error of K and V after
    :func:`quantize_fp8_kv`, their worst per-(token, head) error, and the bytes before /
    after (codes + one fp32 scale per token and head)."""
    from .quant import _pair_stats

    report: dict[str, Any] = {"format": "float8_e4m3fn", "granularity": "per token and head"}
    for name, t in (("k", k), ("v", v)):
        a = t.detach().float()
        st = _pair_stats(a, dequantize_fp8_kv(*quantize_fp8_kv(a)))  # one pass: row sums
        rows = st[:, 2].sqrt() / st[:, 0].sqrt().clamp_min(1e-30)
        norm, err, worst = torch.stack([st[:, 0].sum().sqrt(), st[:, 2].sum().sqrt(),
                                        rows.max() if rows.numel() else st.new_zeros(())]).tolist()
        report[f"{name}_rel_l2"] = round(err / norm, 5) if norm else 0.0
        report[f"{name}_worst_row_rel_l2"] = round(worst, 5) if rows.numel() else 0.0
    elems = k.numel() + v.numel()
    rows = elems // max(k.shape[-1], 1)
    report["bytes"] = {"before": elems * k.element_size(), "after": elems + 4 * rows}
    return report


class Fp8KVCache:
    """A preallocated e4m3 KV cache ``[batch, kv_heads, max_tokens, head_dim]`` with one fp32
    scale per (token, head) (kv_quant.py:104-151). :meth:`append` quantises only the new
    tokens, straight into their slots (the same codes as quantising the whole cache at once),
    and returns the valid views."""

    def __init__(self, batch: int, kv_heads: int, max_tokens: int, head_dim: int,
                 device: torch.device | str | None = None) -> None:
        _check_head_dim(head_dim)
        dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        if dev.type != "cuda":
            raise ValueError("CUDA device required (kernel_agent_b200 runs on the GPU only)")
        shape = (batch, kv_heads, max_tokens, head_dim)
        self.k = torch.zeros(shape, dtype=_E4M3, device=dev)
        self.v = torch.zeros(shape, dtype=_E4M3, device=dev)
        self.k_scale = torch.ones(shape[:3], dtype=torch.float32, device=dev)
        self.v_scale = torch.ones(shape[:3], dtype=torch.float32, device=dev)
        self.length = 0

    def append(self, k: torch.Tensor, v: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
        """Write ``k``, ``v`` ``[batch, kv_heads, new, head_dim]`` after the cached tokens;
        returns ``(k_codes, k_scales, v_codes, v_scales)`` of every valid token."""
        start, end = self.length, self.length + k.shape[2]
        if end > self.k.shape[2]:
            raise ValueError(f"FP8 KV cache full: {end} > {self.k.shape[2]} tokens")
        b, hkv, _, d = self.k.shape
        if k.shape != (b, hkv, end - start, d) or v.shape != k.shape:
            raise ValueError(f"expected k and v [{b}, {hkv}, new, {d}]; got {tuple(k.shape)}, {tuple(v.shape)}")
        nat.require_cuda(k, v, self.k)
        new = end - start
        if new:
            lmax = self.k.shape[2]
            for codes, scales, t in ((self.k, self.k_scale, k), (self.v, self.v_scale, v)):
                x = _kv_input(t)
                nat.call("kab_quant_kv_fp8", x.data_ptr(), nat.dtype_code(x), b * hkv, new, d, new * d, d,
                         codes.data_ptr() + start * d, lmax * d, d, scales.data_ptr() + 4 * start, lmax, 1,
                         nat.stream_of(x))
        self.length = end
        return self.k[:, :, :end], self.k_scale[:, :, :end], self.v[:, :, :end], self.v_scale[:, :, :end]


def kv_cache_share(*, batch: int, tokens: int, layers: int, kv_heads: int, head_dim: int, other_bytes: float,
                   elem_bytes: float = 2.0) -> dict[str, float]:
    """The KV cache's share of what one decode step reads (kv_quant.py:154-183): ``kv_bytes``
    (K and V of every layer at ``tokens`` cached tokens), ``share`` of ``kv_bytes +
    other_bytes`` and the step's bytes e4m3 K / V would save (``saved_share``; one fp32 scale
    per token and head included)."""
    rows = 2 * batch * tokens * layers * kv_heads
    kv = rows * head_dim * elem_bytes
    fp8 = rows * (head_dim + 4)
    total = kv + other_bytes
    return {
        "kv_bytes": kv,
        "share": kv / total if total else 0.0,
        "saved_share": max(kv - fp8, 0.0) / total if total else 0.0,
    }


# ------------------------------------------------------------------ the example's module


def _decode_ok(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> bool:
    """triton_fp8_kv_decode.py:263-276: the shapes the kernel takes."""
    if q.dim() != 4 or k.dim() != 4 or q.shape[2] != 1 or k.shape != v.shape:
        return False
    b, hq, _, d = q.shape
    return (k.shape[0] == b and k.shape[3] == d and k.shape[2] >= 1 and hq % k.shape[1] == 0
            and d in (64, 128) and hq // k.shape[1] <= 32)


class Fp8KVDecodeAttention(nn.Module):
    """SDPA decode attention (``q [B, Hq, 1, D]``, ``k / v [B, Hkv, L, D]``) reading K / V in
    e4m3 with per-(token, head) scales (triton_fp8_kv_decode.py:279-296). Here K and V are
    quantised on every call so that the result can be checked; in a model the cache is
    written in e4m3 when tokens are appended (:class:`Fp8KVCache`) and
    :func:`fp8_kv_decode` reads it."""

    def __init__(self, reference: nn.Module) -> None:
        super().__init__()
        self.reference = reference
        self.scale = getattr(reference, "scale", None)

    def forward(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
        if not _decode_ok(q, k, v):
            raise NotImplementedError(
                f"FP8 KV decode: q {tuple(q.shape)}, k {tuple(k.shape)}: the kernel takes q [B, Hq, 1, D] with "
                "D 64 or 128 and at most 32 query heads per KV head")
        kc, ks = quantize_kv(k)
        vc, vs = quantize_kv(v)
        out = fp8_kv_decode(q, kc, ks, vc, vs, self.scale)
        return out if q.dtype == torch.bfloat16 else out.to(q.dtype)


def build(reference: nn.Module) -> nn.Module:
    return Fp8KVDecodeAttention(reference)
