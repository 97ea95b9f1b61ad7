"""Generate the golden error reports that pin the oracle's report restatements
(``oracle/reports.py``) and the GPU mirror's reports.

Run in a container where the reference sources are present (they are not on the GPU box):

    python tests/golden/make_golden_reports.py /path/to/kernel-agent/src

It imports the reference's own ``kernel_agent.kernels.quant``, runs its error reports
(``fp8_error``, ``int8_error``, ``fp4_error``, ``mxfp8_error``, ``fp8_w8a8_error``,
``int8_w8a8_error``, ``fp4_w4a4_error``, ``fp4_saturation``, ``smoothquant_factors``) on seeded
inputs and writes ``reports_golden.npz`` (the inputs: bf16 as uint16 bits) and
``reports_golden.json`` (the reports). The fixtures are committed; the tests only read them.
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


def main(src: str) -> None:
    sys.path.insert(0, src)
    from kernel_agent.kernels import quant  # noqa: E402  (the reference)

    bf = torch.bfloat16
    g = torch.Generator().manual_seed(20)
    out: dict[str, np.ndarray] = {}
    rep: dict[str, object] = {}
    for name, n in (("w128", 128), ("w48", 48)):
        w = (torch.randn(n, 256, generator=g) * 0.05).to(bf)
        w[3, 17] = 1.5  # an outlier: high crest, underflow in its row
        w[5] = 0  # a zero row
        out[name] = bits(w)
    x = torch.randn(40, 256, generator=g)
    x[:, 9] *= 30.0  # an outlier channel
    x = x.to(bf)
    out["x"] = bits(x)
    w, w48 = (torch.from_numpy(out[k].view(np.int16)).view(bf) for k in ("w128", "w48"))

    rep["fp8_error"] = quant.fp8_error(w, *quant.quantize_fp8(w))
    rep["fp8_error_x"] = quant.fp8_error(w, *quant.quantize_fp8(w), x)
    rep["int8_error"] = quant.int8_error(w, *quant.quantize_int8(w))
    rep["int8_error_x"] = quant.int8_error(w48, *quant.quantize_int8(w48), x)
    rep["fp4_error_nv_x"] = quant.fp4_error(w, *quant.quantize_fp4(w, "nvfp4"), x)
    rep["fp4_error_mx"] = quant.fp4_error(w48, *quant.quantize_fp4(w48, "mxfp4"))
    rep["fp4_error_unbiased"] = quant.fp4_error(w, *quant.quantize_fp4(w, "nvfp4", unbiased=True))
    rep["mxfp8_error"] = quant.mxfp8_error(w, *quant.quantize_mxfp8(w))
    rep["mxfp8_error_x"] = quant.mxfp8_error(w, *quant.quantize_mxfp8(w), x)
    rep["mxfp8_error_x48"] = quant.mxfp8_error(w48, *quant.quantize_mxfp8(w48), x)
    rep["fp8_w8a8_error"] = quant.fp8_w8a8_error(w, *quant.quantize_fp8(w), x)
    rep["int8_w8a8_error"] = quant.int8_w8a8_error(w, *quant.quantize_int8(w), x)
    s = quant.smoothquant_factors(x.float().abs().amax(dim=0), w, 0.4)
    out["smooth"] = s.numpy()
    rep["int8_w8a8_error_smooth"] = quant.int8_w8a8_error(w, *quant.quantize_int8(w, s), x, smooth=s)
    rep["fp4_w4a4_error"] = quant.fp4_w4a4_error(w, *quant.quantize_fp4(w), x)
    rep["fp4_w4a4_error_tensor"] = quant.fp4_w4a4_error(w, *quant.quantize_fp4(w), x, granularity="tensor")
    wr = quant.hadamard_rotate(w.float(), 32)
    rep["fp4_w4a4_error_rot"] = quant.fp4_w4a4_error(w, *quant.quantize_fp4(wr), x, rotate=32)
    rep["fp4_w4a4_error_unbiased"] = quant.fp4_w4a4_error(w, *quant.quantize_fp4(w, unbiased=True), x,
                                                          unbiased=True)
    rep["fp4_w4a4_error_mx"] = quant.fp4_w4a4_error(w, *quant.quantize_fp4(w, "mxfp4"), x, fmt="mxfp4")
    stress = quant.fp4_stress_input((64, 256), "nvfp4", seed=3)
    out["stress"] = bits(stress.to(bf))
    xq, xs, outer = quant.quantize_fp4_activations(stress.to(bf), "nvfp4")
    rep["fp4_saturation"] = quant.fp4_saturation(stress.to(bf), xs, outer)
    rep["fp4_saturation_plain"] = quant.fp4_saturation(x, *quant.quantize_fp4_activations(x)[1:])

    np.savez_compressed(HERE / "reports_golden.npz", **out)
    (HERE / "reports_golden.json").write_text(json.dumps(rep, indent=1, sort_keys=True) + "\n")
    print(f"wrote {len(out)} arrays, {len(rep)} reports")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit(f"usage: python {sys.argv[0]} <path to the reference's src directory>")
    main(sys.argv[1])
