"""The tcgen05 scaled GEMMs of ``libkab.so`` (``kab_gemm_*``), called by the linears of
:mod:`kernel_agent_b200.kernels.quant` and :mod:`kernel_agent_b200.kernels.blockwise`.

Operands are K-major codes (``A [M, K]``, ``B [N, K]``, the ``nn.Linear`` weight layout);
block scales are passed in the swizzled 128 x 4 layout. The kernels need whole 128-byte
k-steps (K a multiple of 128 for 8-bit codes, 256 for FP4) and, block-scaled, N a multiple of
128; other shapes are zero-padded here (zero codes with zero scales add nothing).
"""

from __future__ import annotations

import ctypes

import torch

from .. import _native as nat

_OUT = {torch.bfloat16: nat.KAB_BF16, torch.float16: nat.KAB_F16, torch.float32: nat.KAB_F32}


def _bind() -> None:
    """The signatures are declared in ``_native``; loading binds them."""
    nat.load()


def _pad_k(t: torch.Tensor, mult: int) -> torch.Tensor:
    k = t.shape[1]
    if k % mult == 0:
        return t.contiguous()
    out = torch.zeros(t.shape[0], k + (-k % mult), dtype=t.dtype, device=t.device)
    out[:, :k] = t
    return out


def _bias(bias: torch.Tensor | None, n: int, device) -> tuple[torch.Tensor | None, int]:
    if bias is None:
        return None, nat.KAB_F32
    b = bias.detach().to(device).reshape(-1)
    if b.numel() != n:
        raise ValueError(f"bias has {b.numel()} elements, expected {n}")
    if b.dtype not in nat.DTYPES:
        b = b.float()
    return b.contiguous(), nat.dtype_code(b)


def _out_code(dtype: torch.dtype) -> tuple[torch.dtype, int]:
    return (dtype, _OUT[dtype]) if dtype in _OUT else (torch.float32, nat.KAB_F32)


def int8(a: torch.Tensor, b: torch.Tensor, a_scale=None, b_scale=None, bias=None,
         out_dtype: torch.dtype | None = None) -> torch.Tensor:
    """int8 ``a [M, K] @ b [N, K]ᵀ``: exact int32 when no scales are given, else the
    epilogue ``acc * a_scale[m] * b_scale[n] (+ bias)`` in ``out_dtype``."""
    _bind()
    m, n = a.shape[0], b.shape[0]
    a2, b2 = _pad_k(a.view(torch.int8), 128), _pad_k(b.view(torch.int8), 128)
    k = a2.shape[1]
    ldo = n + (-n % 8)
    if a_scale is None:
        acc = torch.empty(m, ldo, dtype=torch.int32, device=a.device)
        nat.call("kab_gemm_i8", a2.data_ptr(), b2.data_ptr(), m, n, k, None, None, None, 0, None,
                 nat.KAB_BF16, ldo, acc.data_ptr(), nat.stream_of(a))
        return acc[:, :n] if ldo != n else acc
    odt, code = _out_code(out_dtype or torch.bfloat16)
    out = torch.empty(m, ldo, dtype=odt, device=a.device)
    bb, bcode = _bias(bias, n, a.device)
    sa, sb = a_scale.float().contiguous(), b_scale.float().to(a.device).contiguous()
    nat.call("kab_gemm_i8", a2.data_ptr(), b2.data_ptr(), m, n, k, sa.data_ptr(), sb.data_ptr(),
             nat.ptr(bb), bcode, out.data_ptr(), code, ldo, None, nat.stream_of(a))
    return out[:, :n] if ldo != n else out


def fp8(a: torch.Tensor, b: torch.Tensor, a_scale, b_scale, bias=None, out_dtype=torch.bfloat16) -> torch.Tensor:
    """e4m3 ``a [M, K] @ b [N, K]ᵀ * a_scale[m] * b_scale[n] (+ bias)``, fp32 accumulation."""
    _bind()
    m, n = a.shape[0], b.shape[0]
    a2, b2 = _pad_k(a.view(torch.uint8), 128), _pad_k(b.view(torch.uint8), 128)
    ldo = n + (-n % 8)
    odt, code = _out_code(out_dtype)
    out = torch.empty(m, ldo, dtype=odt, device=a.device)
    bb, bcode = _bias(bias, n, a.device)
    sa, sb = a_scale.float().contiguous(), b_scale.float().to(a.device).contiguous()
    nat.call("kab_gemm_f8", a2.data_ptr(), b2.data_ptr(), m, n, a2.shape[1], sa.data_ptr(), sb.data_ptr(),
             nat.ptr(bb), bcode, out.data_ptr(), code, ldo, nat.stream_of(a))
    return out[:, :n] if ldo != n else out


def mxf8(a: torch.Tensor, a_sf_swizzled: torch.Tensor, b: torch.Tensor, b_sf_swizzled: torch.Tensor,
         bias=None, out_dtype=torch.bfloat16) -> torch.Tensor:
    """MXFP8 ``a [M, K] @ b [N, K]ᵀ`` with e8m0 scales per 32 (swizzled) applied by the tensor
    core; the result in ``out_dtype``, then ``+ bias`` in that dtype. K % 128 == 0, N % 128 == 0."""
    _bind()
    m, n, k = a.shape[0], b.shape[0], a.shape[1]
    if k % 128:
        raise ValueError(f"the MXFP8 GEMM needs K a multiple of 128 (got {k})")
    odt, code = _out_code(out_dtype)
    ldo = n + (-n % 8)
    out = torch.empty(m, ldo, dtype=odt, device=a.device)
    bb, bcode = _bias(bias, n, a.device)
    nat.call("kab_gemm_mxf8", a.contiguous().data_ptr(), a_sf_swizzled.data_ptr(), b.contiguous().data_ptr(),
             b_sf_swizzled.data_ptr(), m, n, k, nat.ptr(bb), bcode, out.data_ptr(), code, ldo, nat.stream_of(a))
    return out[:, :n] if ldo != n else out


def nvf4(a: torch.Tensor, a_sf_swizzled: torch.Tensor, a_outer: torch.Tensor, b: torch.Tensor,
         b_sf_swizzled: torch.Tensor, b_scale: torch.Tensor, bias=None, out_dtype=torch.bfloat16,
         out: torch.Tensor | None = None, peer_out: list[int] | None = None) -> torch.Tensor:
    """NVFP4 ``a [M, K/2] @ b [N, K/2]ᵀ`` (packed e2m1) with e4m3 scales per 16 (swizzled)
    applied by the tensor core, then ``acc * (a_outer[m] * b_scale) (+ bias)``; ``b_scale``:
    one value or one per row of b. K % 256 == 0. ``out``: an optional ``[M, N]`` destination
    (a column block of a wider buffer: its row stride is used). ``peer_out``: device addresses
    (other ranks' buffers mapped by CUDA IPC) of the same block in buffers of the same layout,
    which the epilogue also writes over NVLink."""
    _bind()
    m, n, k = a.shape[0], b.shape[0], 2 * a.shape[1]
    if k % 256:
        raise ValueError(f"the NVFP4 GEMM needs K a multiple of 256 (got {k})")
    odt, code = _out_code(out_dtype)
    if out is None:
        ldo = n + (-n % 8)
        full = torch.empty(m, ldo, dtype=odt, device=a.device)
        out = full[:, :n]
    elif out.shape != (m, n) or out.stride(1) != 1 or out.dtype != odt:
        raise ValueError("out must be [M, N] with unit column stride in the output dtype")
    bb, bcode = _bias(bias, n, a.device)
    ts = b_scale.float().to(a.device).reshape(-1).contiguous()
    per_col = int(ts.numel() > 1)
    if per_col and ts.numel() != n:
        raise ValueError(f"b_scale has {ts.numel()} values, expected 1 or {n}")
    args = (a.contiguous().data_ptr(), a_sf_swizzled.data_ptr(), a_outer.float().contiguous().data_ptr(),
            b.contiguous().data_ptr(), b_sf_swizzled.data_ptr(), ts.data_ptr(), per_col, m, n, k, nat.ptr(bb), bcode,
            out.data_ptr(), code, out.stride(0))
    if peer_out:
        arr = (ctypes.c_void_p * len(peer_out))(*peer_out)
        nat.call("kab_gemm_nvf4_scatter", *args, arr, len(peer_out), nat.stream_of(a))
    else:
        nat.call("kab_gemm_nvf4", *args, nat.stream_of(a))
    return out


def mxf4(a: torch.Tensor, a_sf_swizzled: torch.Tensor, b: torch.Tensor, b_sf_swizzled: torch.Tensor,
         b_scale: torch.Tensor | None = None, bias=None, out_dtype=torch.bfloat16,
         a_outer: torch.Tensor | None = None) -> torch.Tensor:
    """MXFP4 ``a [M, K/2] @ b [N, K/2]ᵀ`` (packed e2m1) with e8m0 scales per 32 (swizzled)
    applied by the tensor core, then ``acc * (outer[m] * ts) (+ bias)``; ``a_outer``: None (1)
    or one per row of a; ``b_scale``: None (1), one value or one per row of b. K % 256 == 0."""
    _bind()
    m, n, k = a.shape[0], b.shape[0], 2 * a.shape[1]
    if k % 256:
        raise ValueError(f"the MXFP4 GEMM needs K a multiple of 256 (got {k})")
    odt, code = _out_code(out_dtype)
    ldo = n + (-n % 8)
    out = torch.empty(m, ldo, dtype=odt, device=a.device)
    bb, bcode = _bias(bias, n, a.device)
    ts, per_col = None, 0
    if b_scale is not None:
        ts = b_scale.float().to(a.device).reshape(-1).contiguous()
        per_col = int(ts.numel() > 1)
        if per_col and ts.numel() != n:
            raise ValueError(f"b_scale has {ts.numel()} values, expected 1 or {n}")
    outer = None if a_outer is None else a_outer.float().reshape(-1).contiguous()
    nat.call("kab_gemm_mxf4", a.contiguous().data_ptr(), a_sf_swizzled.data_ptr(), nat.ptr(outer),
             b.contiguous().data_ptr(), b_sf_swizzled.data_ptr(), nat.ptr(ts), per_col, m, n, k, nat.ptr(bb), bcode,
             out.data_ptr(), code, ldo, nat.stream_of(a))
    return out[:, :n] if ldo != n else out


def fp8_blockwise(a: torch.Tensor, a_scale: torch.Tensor, b: torch.Tensor, b_scale: torch.Tensor, bias=None,
                  out_dtype=torch.bfloat16) -> torch.Tensor:
    """Blockwise FP8 ``a [M, K] @ b [N, K]ᵀ``: ``a_scale [M, K/128]`` per 1 x 128 group,
    ``b_scale [N/128, K/128]`` per 128 x 128 block, promoted per 128-wide K step in fp32
    (+ bias), one rounding to ``out_dtype``. K % 128 == 0, N % 128 == 0."""
    _bind()
    m, k = a.shape
    n = b.shape[0]
    if b.shape[1] != k:
        raise ValueError(f"K mismatch: a has {k}, b has {b.shape[1]}")
    if k % 128 or n % 128:
        raise ValueError(f"the blockwise GEMM needs K and N multiples of 128 (got K={k}, N={n})")
    if tuple(a_scale.shape) != (m, k // 128) or tuple(b_scale.shape) != (n // 128, k // 128):
        raise ValueError(f"scales {tuple(a_scale.shape)} / {tuple(b_scale.shape)} do not match "
                         f"[{m}, {k // 128}] / [{n // 128}, {k // 128}]")
    odt, code = _out_code(out_dtype)
    ldo = n + (-n % 8)
    out = torch.empty(m, ldo, dtype=odt, device=a.device)
    bb, bcode = _bias(bias, n, a.device)
    sa = a_scale.float().contiguous()
    sb = b_scale.float().to(a.device).contiguous()
    nat.call("kab_gemm_f8_blockwise", a.contiguous().view(torch.uint8).data_ptr(), sa.data_ptr(),
             b.contiguous().view(torch.uint8).data_ptr(), sb.data_ptr(), m, n, k, nat.ptr(bb), bcode,
             out.data_ptr(), code, ldo, nat.stream_of(a))
    return out[:, :n] if ldo != n else out
