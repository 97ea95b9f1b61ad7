"""Conversions between torch tensors and the oracle's numpy arrays (tests only)."""

from __future__ import annotations

import numpy as np
import torch

from oracle.formats import bf16_to_f32


def np_values(t: torch.Tensor) -> np.ndarray:
    """fp32 numpy values of a float tensor (bf16 / fp16 / fp32), any device."""
    t = t.detach().cpu().contiguous()
    if t.dtype == torch.bfloat16:
        return bf16_to_f32(t.view(torch.int16).numpy().view(np.uint16))
    return t.float().numpy()


def np_bytes(t: torch.Tensor) -> np.ndarray:
    """The raw bytes of a tensor as uint8 (fp8 / e8m0 / uint8 / int8), any device."""
    t = t.detach().cpu().contiguous()
    if t.dtype in (torch.float8_e4m3fn, torch.float8_e8m0fnu, torch.int8):
        t = t.view(torch.uint8)
    return t.numpy()


def np_bf16_bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def to_bf16(a: np.ndarray, device="cuda") -> torch.Tensor:
    """A bf16 tensor holding fp32 values ``a`` that are bf16-representable."""
    t = torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32))
    return t.to(torch.bfloat16).to(device)


def bits_to_bf16(bits: np.ndarray, device="cuda") -> torch.Tensor:
    t = torch.from_numpy(np.ascontiguousarray(bits, dtype=np.uint16).view(np.int16))
    return t.view(torch.bfloat16).to(device)


def ulp_distance_bf16(a_bits: np.ndarray, b_bits: np.ndarray) -> np.ndarray:
    """|a - b| in bf16 steps (sign-magnitude mapped to a monotonic line)."""
    a = a_bits.astype(np.int32)
    b = b_bits.astype(np.int32)
    a = np.where(a & 0x8000, -(a & 0x7FFF), a)
    b = np.where(b & 0x8000, -(b & 0x7FFF), b)
    return np.abs(a - b)
