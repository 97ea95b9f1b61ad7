"""The reference's CPU execution path of each benchmarked workload (test infrastructure:
``bench.py``'s CPU legs time it; ``tests/test_oracle_cpu_path.py`` checks it against the
exact restatements of ``oracle.quant`` / ``oracle.fp8lib``).

Where the reference runs a GEMM on the CPU it calls torch's fp32 matmul (MKL / OpenBLAS
sgemm on every core): ``fp4_w4a4_linear`` ``fp4_values(xq, xs) @ fp4_values(codes, scales).T``
(``src/kernel_agent/kernels/quant.py:1247-1248``), ``mxfp8_linear`` on the dequantised
operands (``quant.py:615-617``), ``int8_matmul`` in fp32 chunks of K = 1024 summed in int32
(``quant.py:881-884``, exact), and the research scripts' blockwise GEMM and qkpv attention on
fake-quantised fp32 tensors (``docs/research-scripts/fp8-sm120/fp8lib.py:22-40, 184-215``,
``gemm_bench.py:39-68``). The restatements in ``oracle.quant`` accumulate in float64 (the
exact value the GPU is judged against); these keep the reference's fp32 arithmetic and call the
same CPU BLAS it does (torch's fp32 matmul), so the timed CPU baseline does the work the
reference's CPU path does. The quantisers are ``oracle.quant``'s (numpy, the same element-wise
fp32 steps as the reference's torch)."""

from __future__ import annotations

import numpy as np
import torch

from . import fp8lib
from . import quant as oq
from .formats import F32, e4m3_to_f32, f32

INT8_EXACT_K = 1024  # quant.py:851: fp32 partial sums of int8 products over 1024 are exact


_E2M1_BYTE_PAIRS = None


def _fp4_values_t(codes, scales, fmt: str) -> torch.Tensor:
    """quant.py:1110-1114 ``fp4_values`` on the host's threads (torch CPU ops): the exact fp32
    values ``e2m1 x block scale`` of packed codes ``[rows, K / 2]``, by table lookups (both
    nibbles of a byte at once, then the 256 e4m3 / e8m0 scale bytes)."""
    global _E2M1_BYTE_PAIRS
    if _E2M1_BYTE_PAIRS is None:
        nib = torch.from_numpy(oq.e2m1_to_f32(np.arange(16)))
        _E2M1_BYTE_PAIRS = torch.stack([nib.repeat(16), nib.repeat_interleave(16)], dim=1)  # [256, 2]
    c = torch.from_numpy(np.ascontiguousarray(codes, np.uint8)).long()
    rows, half = c.shape
    vals = _E2M1_BYTE_PAIRS[c].reshape(rows, 2 * half)
    table = oq.e4m3_to_f32(np.arange(256)) if fmt == "nvfp4" else oq.e8m0_to_f32(np.arange(256))
    sc = torch.from_numpy(table)[torch.from_numpy(np.ascontiguousarray(scales, np.uint8)).long()]
    nb = sc.shape[1]
    return (vals.reshape(rows, nb, -1) * sc[:, :, None]).reshape(rows, 2 * half)


def sgemm_nt(a, b) -> np.ndarray:
    """``a @ bᵀ`` in fp32 through torch's CPU matmul (the BLAS the reference's CPU path calls,
    on every host thread)."""
    ta = a if isinstance(a, torch.Tensor) else torch.from_numpy(np.ascontiguousarray(a, F32))
    tb = b if isinstance(b, torch.Tensor) else torch.from_numpy(np.ascontiguousarray(b, F32))
    return (ta @ tb.T).numpy()


def int8_matmul(a, b) -> np.ndarray:
    """quant.py:881-884: int32 ``a @ bᵀ`` as fp32 matmuls over chunks of K = 1024 (each partial
    sum an exact integer), summed in int32."""
    a, b = np.asarray(a, np.int8), np.asarray(b, np.int8)
    acc = np.zeros((a.shape[0], b.shape[0]), np.int32)
    for k0 in range(0, a.shape[1], INT8_EXACT_K):
        part = sgemm_nt(a[:, k0:k0 + INT8_EXACT_K].astype(F32), b[:, k0:k0 + INT8_EXACT_K].astype(F32))
        acc += part.astype(np.int32)
    return acc


def int8_w8a8_linear(x, q, scale, bias=None) -> np.ndarray:
    """quant.py:901-923 on the CPU: per-token int8 activations, the fp32-chunk product, the
    fp32 epilogue; bf16 bits."""
    xq, xs = oq.quantize_int8_activations(x)
    return oq.to_dtype(oq.int8_epilogue(int8_matmul(xq, q), xs, scale, bias), "bf16")


def fp4_w4a4_linear(x, codes, scales, ts, bias=None, fmt="nvfp4", granularity="token") -> np.ndarray:
    """quant.py:1233-1257 on the CPU: activations quantised per call, the fp32 matmul of the
    exact block-scaled values, ``acc * (outer * ts) (+ bias)``; bf16 bits."""
    xq, xs, outer = oq.quantize_fp4_activations(x, fmt, granularity)
    acc = sgemm_nt(_fp4_values_t(xq, xs, fmt), _fp4_values_t(codes, scales, fmt))
    return oq.to_dtype(oq.fp4_epilogue(acc.astype(F32), outer, ts, bias), "bf16")


def mxfp8_linear_codes(xq, xs, q, scales, bias=None) -> np.ndarray:
    """quant.py:615-619 on the CPU, from already quantised activations: the fp32 matmul of the
    dequantised operands (+ bias); bf16 bits."""
    y = sgemm_nt(oq.dequantize_mxfp8(xq, xs), oq.dequantize_mxfp8(q, scales))
    if bias is not None:
        y = (y + f32(bias)[None, :]).astype(F32)
    return oq.to_dtype(y, "bf16")


def silu_mul_mxfp8(gate, up) -> tuple[np.ndarray, np.ndarray]:
    """The config-3 producer on the CPU: ``F.silu(gate) * up`` in bf16 (its two roundings),
    then quantize_mxfp8 (quant.py:506-526)."""
    return oq.quantize_mxfp8(oq.silu_mul(gate, up))


def fp8_blockwise_linear(x, wq, ws, group: int = 128) -> np.ndarray:
    """fp8lib.py:22-40 / gemm_bench.py:39-68 on the CPU: the activations fake-quantised per
    1 x 128 group, then ``(codes * sa) @ (codes * sb)ᵀ`` in fp32; bf16 bits."""
    xq, xs = fp8lib.quantize_fp8_groups(x, group)
    a = (e4m3_to_f32(xq).reshape(xq.shape[0], -1, group) * xs[:, :, None]).reshape(xq.shape).astype(F32)
    n, k = wq.shape
    wsf = np.repeat(np.repeat(f32(ws), group, axis=0)[:n], group, axis=1)[:, :k]
    b = (e4m3_to_f32(wq) * wsf).astype(F32)
    return oq.to_dtype(sgemm_nt(a, b), "bf16")


def attention_fp8_head(q, k, v, causal: bool = True) -> np.ndarray:
    """fp8lib.py:184-215 (``emulated_sdpa`` mode qkpv) for one (batch, head) in fp32 as the
    research script runs it on torch: fake-quantised Q, K, V, fp32 scores and softmax, P as
    ``e4m3(p * 448) / 448``, fp32 ``P V``."""
    qc, qs = fp8lib.quantize_head(q)
    kc, ks = fp8lib.quantize_head(k)
    vc, vs = fp8lib.quantize_head(v)
    qf, kf, vf = ((e4m3_to_f32(c) * s).astype(F32) for c, s in ((qc, qs), (kc, ks), (vc, vs)))
    s = sgemm_nt(qf, kf) * F32(qf.shape[-1] ** -0.5)
    if causal:
        s = np.where(np.triu(np.ones(s.shape, bool), 1), -np.inf, s).astype(F32)
    p = np.exp(s - s.max(axis=-1, keepdims=True)).astype(F32)
    denom = p.sum(axis=-1, keepdims=True, dtype=F32)
    p8 = (e4m3_to_f32(fp8lib.q8_codes((p * F32(fp8lib.FMAX)).astype(F32))) / F32(fp8lib.FMAX)).astype(F32)
    return (sgemm_nt(p8, np.ascontiguousarray(vf.T)) / denom).astype(F32)
