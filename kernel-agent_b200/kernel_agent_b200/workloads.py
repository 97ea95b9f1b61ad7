"""Seeded synthetic inputs of the five benchmark configurations.

The reference's calibration captures are not available, so these stand in for them with
the shapes and value distributions the configurations name. ``device="cpu"`` draws with a
CPU ``torch.Generator`` (the same bits on every machine with this torch, used by the parity
tests); ``device="cuda"`` draws on the GPU (the benchmark's full-size inputs).

1. W8A8 INT8: X [128, 1024] N(0, 1) with 5 of 1024 columns (0.5 %) x 20, W [1024, 1024]
   N(0, 0.02), bias [1024] N(0, 0.1).
2. FP8 blockwise: X [M, 1024] N(0, 1), M in {1, 16, 2048}; W [3072, 1024] N(0, 0.02) with
   1 % of the entries replaced by Student-t(nu = 3) x 0.02.
3. MXFP8 MLP: gate, up [4096, 14336] N(0, 1); W_down [4096, 14336] N(0, 0.015).
4. W4A4 NVFP4: X [8192, 8192] N(0, 1) with 16 of 8192 columns (0.2 %) x 30,
   W [28672, 8192] N(0, 0.01), bias [28672] N(0, 0.05).
5. FP8 attention: Q [4, 32, 4096, 128], K / V [4, 8, 4096, 128] N(0, 1).
All bf16.
"""

from __future__ import annotations

import torch

BF16 = torch.bfloat16


def _gen(seed: int, device: str) -> torch.Generator:
    return torch.Generator(device=device).manual_seed(seed)


def _randn(shape, g, device, std: float = 1.0) -> torch.Tensor:
    return torch.randn(*shape, generator=g, device=device) * std


def _outlier_columns(x: torch.Tensor, count: int, factor: float, g) -> torch.Tensor:
    cols = torch.randperm(x.shape[1], generator=g, device=g.device)[:count]
    x[:, cols] *= factor
    return x


def config1(seed: int = 0, device: str = "cpu", m: int = 128, k: int = 1024, n: int = 1024):
    """(x, w, bias) of configuration 1."""
    g = _gen(seed, device)
    x = _outlier_columns(_randn((m, k), g, device), max(1, round(0.005 * k)), 20.0, g)
    w = _randn((n, k), g, device, 0.02)
    b = _randn((n,), g, device, 0.1)
    return x.to(BF16), w.to(BF16), b.to(BF16)


def config2(m: int, seed: int = 0, device: str = "cpu", k: int = 1024, n: int = 3072):
    """(x, w) of configuration 2 (a weight with 1 % Student-t(3) entries)."""
    g = _gen(seed, device)
    x = _randn((m, k), g, device)
    w = _randn((n, k), g, device, 0.02)
    heavy = torch.rand(n, k, generator=g, device=device) < 0.01
    z = _randn((n, k), g, device)
    chi2 = sum(_randn((n, k), g, device) ** 2 for _ in range(3))
    t = z / torch.sqrt(chi2 / 3.0)
    w = torch.where(heavy, t * 0.02, w)
    return x.to(BF16), w.to(BF16)


def config3(seed: int = 0, device: str = "cpu", m: int = 4096, f: int = 14336, h: int = 4096):
    """(gate, up, w_down) of configuration 3."""
    g = _gen(seed, device)
    gate = _randn((m, f), g, device).to(BF16)
    up = _randn((m, f), g, device).to(BF16)
    w = _randn((h, f), g, device, 0.015).to(BF16)
    return gate, up, w


def config4(seed: int = 0, device: str = "cpu", m: int = 8192, k: int = 8192, n: int = 28672):
    """(x, w, bias) of configuration 4."""
    g = _gen(seed, device)
    x = _outlier_columns(_randn((m, k), g, device), max(1, round(0.002 * k)), 30.0, g)
    w = _randn((n, k), g, device, 0.01)
    b = _randn((n,), g, device, 0.05)
    return x.to(BF16), w.to(BF16), b.to(BF16)


def config5(seed: int = 0, device: str = "cpu", b: int = 4, hq: int = 32, hkv: int = 8,
            s: int = 4096, d: int = 128):
    """(q, k, v) of configuration 5."""
    g = _gen(seed, device)
    q = _randn((b, hq, s, d), g, device).to(BF16)
    k = _randn((b, hkv, s, d), g, device).to(BF16)
    v = _randn((b, hkv, s, d), g, device).to(BF16)
    return q, k, v
