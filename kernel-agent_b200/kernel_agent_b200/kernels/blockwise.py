"""Blockwise FP8 (1 x 128 activation groups, 128 x 128 weight blocks): a new API in the
style of ``kernel_agent.kernels.quant``.

The toolkit has no blockwise recipe; its math is the reference's research fake-quant
(``docs/research-scripts/fp8-sm120/fp8lib.py:22-40``: ``fq_groups``, ``fq_block``; one scale
``amax / 448`` per group or block, a zero scale replaced by 1, e4m3 codes to nearest even)
and the blockwise GEMM's promotion rule (``docs/research-scripts/fp8-sm120/gemm_bench.py:
39-68``: a fresh fp32 partial product per 128-wide K step, multiplied by both scales and
added into the fp32 accumulator).
"""

from __future__ import annotations

import torch

from .. import _native as nat
from . import quant as q

GROUP = 128
_E4M3 = torch.float8_e4m3fn


def quantize_fp8_groups(x: torch.Tensor, group: int = GROUP) -> tuple[torch.Tensor, torch.Tensor]:
    """``(codes e4m3 [rows, K], scales fp32 [rows, K / group])`` of ``x [..., K]``: one scale
    per 1 x ``group`` along K (fp8lib.py:22-27). ``group``: 32, 64 or 128."""
    k = x.shape[-1]
    if group not in (32, 64, 128):
        raise ValueError(f"group {group} is not 32, 64 or 128")
    if k % group:
        raise ValueError(f"the last dimension {k} is not a multiple of the group ({group})")
    nat.require_cuda(x)
    x2 = q._rows(q._input(x))
    m = x2.shape[0]
    codes = torch.empty(m, k, dtype=_E4M3, device=x2.device)
    scales = torch.empty(m, k // group, dtype=torch.float32, device=x2.device)
    if m and k:
        nat.call("kab_quant_groups_fp8", x2.data_ptr(), nat.dtype_code(x2), m, k, x2.stride(0), group,
                 codes.data_ptr(), scales.data_ptr(), nat.stream_of(x2))
    return codes, scales


def quantize_fp8_blocks(weight: torch.Tensor, block: int = GROUP) -> tuple[torch.Tensor, torch.Tensor]:
    """``(codes e4m3 [N, K], scales fp32 [N / 128, K / 128])`` of a 2-D weight: one scale per
    128 x 128 block (fp8lib.py:35-39)."""
    if weight.dim() != 2:
        raise ValueError(f"expected a 2-D weight [out, in], got shape {tuple(weight.shape)}")
    if block != GROUP:
        raise ValueError(f"block {block} is not 128 (the blockwise recipe's block)")
    n, k = weight.shape
    if n % block or k % block:
        raise ValueError(f"weight {tuple(weight.shape)} is not a whole number of {block} x {block} blocks")
    nat.require_cuda(weight)
    w = q._rows(q._input(weight))
    codes = torch.empty(n, k, dtype=_E4M3, device=w.device)
    scales = torch.empty(n // block, k // block, dtype=torch.float32, device=w.device)
    if n and k:
        nat.call("kab_quant_blocks_fp8", w.data_ptr(), nat.dtype_code(w), n, k, w.stride(0),
                 codes.data_ptr(), scales.data_ptr(), nat.stream_of(w))
    return codes, scales


def fp8_blockwise_linear(x: torch.Tensor, codes: torch.Tensor, scales: torch.Tensor, bias=None,
                         out_dtype: torch.dtype | None = None) -> torch.Tensor:
    """``x [..., K] @ Wᵀ`` with W given as blockwise FP8 (``codes [N, K]`` e4m3, ``scales
    [N/128, K/128]`` fp32 from :func:`quantize_fp8_blocks`): ``x`` is quantised per 1 x 128
    group, the tcgen05 GEMM promotes each 128-wide K step in fp32 (gemm_bench.py:39-68), then
    ``+ bias`` and one rounding to ``out_dtype`` (default ``x.dtype``). Returns ``[..., N]``."""
    from . import gemm

    if codes.dim() != 2:
        raise ValueError(f"expected 2-D codes [out, in], got shape {tuple(codes.shape)}")
    n, k = codes.shape
    if x.shape[-1] != k:
        raise ValueError(f"x has {x.shape[-1]} input features, the weight {k}")
    nat.require_cuda(x, codes, scales)
    lead = x.shape[:-1]
    xq, xs = quantize_fp8_groups(x.reshape(-1, k))
    y = gemm.fp8_blockwise(xq, xs, codes, scales, bias=bias, out_dtype=out_dtype or x.dtype)
    return y.reshape(*lead, n)
