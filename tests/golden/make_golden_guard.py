"""Generate the golden scale-guard reports that pin the GPU scale guard
(``kernel_agent_b200.kernels.scale_guard``) to the reference's.

Run in a container where the reference sources are present (they are not on the GPU box):

    python tests/golden/make_golden_guard.py /path/to/kernel-agent/src

It imports the reference's own ``kernel_agent.kernels.scale_guard`` and ``quant``, runs
``outliers`` on seeded activations (outlier channels, zero rows, NaN / inf, bf16 / fp16 / fp32,
K not a multiple of 8) and ``check`` with quantisers built on the reference's quantisers
(the ceil and floor MXFP8 rules, NVFP4 / MXFP4, a truncating NVFP4 scale, a rotating
quantiser, a failing one, a missing one), and writes ``guard_golden.npz`` (the inputs: 2-byte
types as uint16 bits) and ``guard_golden.json`` (the results). The fixtures are committed;
the tests only read them.
"""

from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def bits(t: torch.Tensor) -> np.ndarray:
    t = t.detach().contiguous().cpu()
    if t.dtype in (torch.bfloat16, torch.float16):
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy()


def inputs() -> dict[str, torch.Tensor]:
    g = torch.Generator().manual_seed(31)
    xs: dict[str, torch.Tensor] = {}
    a = torch.randn(96, 512, generator=g)
    a[:, 7] *= 40.0  # a massive-activation channel
    a[:, 300] *= 9.0
    xs["bf16_outlier"] = a.to(torch.bfloat16)
    b = torch.randn(40, 256, generator=g) * 0.01
    b[3] = 0.0  # a zero row: no crest of its own
    b[5, 11] = float("nan")
    b[6, 12] = float("inf")
    b[7, 200] = -float("inf")
    xs["fp16_specials"] = b.to(torch.float16)
    xs["f32_3d"] = torch.randn(2, 24, 160, generator=g) * 3.0
    xs["bf16_odd_k"] = torch.randn(33, 20, generator=g).to(torch.bfloat16)  # K % 8 != 0
    xs["bf16_zero"] = torch.zeros(16, 64, dtype=torch.bfloat16)
    return xs


def main(src: str) -> None:
    sys.path.insert(0, src)
    from kernel_agent.kernels import quant, scale_guard  # noqa: E402  (the reference)

    xs = inputs()
    out = {name: bits(x) for name, x in xs.items()}
    result: dict[str, object] = {"outliers": {name: scale_guard.outliers(x) for name, x in xs.items()}}

    def truncating(t):
        c, s, o = quant.quantize_fp4_activations(t, "nvfp4")
        return c, (torch.floor(s.float() * 8) / 8).to(torch.float8_e4m3fn), o

    def rotating(t):
        r = quant.hadamard_rotate(t, 16)
        c, s, o = quant.quantize_fp4_activations(r, "nvfp4")
        return c, s, o, r

    def failing(t):
        raise RuntimeError("the candidate's quantiser failed")

    hooks = {
        "mx_ceil": ("fp8_mx", lambda t: quant.quantize_mxfp8(t, "ceil")),
        "mx_floor": ("fp8_mx", lambda t: quant.quantize_mxfp8(t, "floor")),
        "nvfp4": ("fp4_w4a4", lambda t: quant.quantize_fp4_activations(t, "nvfp4")),
        "mxfp4": ("fp4_w4a4", lambda t: quant.quantize_fp4_activations(t, "mxfp4")),
        "nvfp4_tensor": ("fp4_w4a4", lambda t: quant.quantize_fp4_activations(t, "nvfp4", "tensor")),
        "truncating": ("fp4_w4a4", truncating),
        "rotating": ("fp4_w4a4", rotating),
        "failing": ("fp8_mx", failing),
        "missing": ("fp4_w4a4", None),
    }
    checks = {}
    x = xs["bf16_outlier"]
    cases = [{"count": 1, "args": (torch.randn(8, 30),)}, {"count": 4, "args": (7, x)}]
    for name, (precision, fn) in hooks.items():
        module = type("Candidate", (), {})()
        if fn is not None:
            module.quantize_activations = fn
        checks[name] = scale_guard.check(module, cases, precision)
    result["checks"] = checks
    result["cases"] = "[{count 1: randn(8, 30)}, {count 4: (7, bf16_outlier)}]"
    np.savez_compressed(HERE / "guard_golden.npz", **out)
    (HERE / "guard_golden.json").write_text(json.dumps(result, indent=1, sort_keys=True) + "\n")
    print(f"wrote {len(out)} inputs, {len(result['outliers'])} outlier reports, {len(checks)} checks")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit(f"usage: python {sys.argv[0]} <path to the reference's src directory>")
    main(sys.argv[1])
