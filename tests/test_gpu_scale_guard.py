"""The GPU scale guard against the reference's own reports (``tests/golden/guard_golden.*``,
made by ``make_golden_guard.py``): the outlier statistics of each input, and whole reports of
``check`` for quantisers of every rule (MXFP8 ceil / floor, NVFP4 per token / per tensor,
MXFP4, a truncating NVFP4 scale, a rotating quantiser, a failing one, a missing one).
Summaries, verdicts, notes and error texts are equal; ``crest`` and ``channel_ratio``, rounded
to one decimal from fp32 sums whose order differs, may differ by that last digit."""

from __future__ import annotations

import json
import types

import numpy as np
import pytest
import torch

from conftest import GOLDEN

pytestmark = pytest.mark.gpu
DEV = "cuda"
DTYPES = {"bf16": torch.bfloat16, "fp16": torch.float16, "f32": torch.float32}


@pytest.fixture(scope="module")
def guard_golden():
    with np.load(GOLDEN / "guard_golden.npz") as z:
        arrays = {k: z[k] for k in z.files}
    return arrays, json.loads((GOLDEN / "guard_golden.json").read_text())


def tensor(name: str, arr: np.ndarray) -> torch.Tensor:
    dtype = DTYPES[name.split("_")[0]]
    if dtype == torch.float32:
        return torch.from_numpy(arr).to(DEV)
    return torch.from_numpy(arr.view(np.int16)).view(dtype).to(DEV)


def same_outliers(got: dict, want: dict, label: str) -> None:
    assert set(got) == set(want), label
    for key in want:
        assert abs(got[key] - want[key]) <= 0.1 + 1e-9, (label, key, got[key], want[key])


def test_outliers(guard_golden):
    from kernel_agent_b200.kernels import scale_guard

    arrays, meta = guard_golden
    for name, want in meta["outliers"].items():
        same_outliers(scale_guard.outliers(tensor(name, arrays[name])), want, name)


def test_check_reports(guard_golden):
    from kernel_agent_b200.kernels import quant, scale_guard

    arrays, meta = guard_golden
    x = tensor("bf16_outlier", arrays["bf16_outlier"])
    cases = [{"count": 1, "args": (torch.randn(8, 30, device=DEV),)}, {"count": 4, "args": (7, x)}]

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
    for name, (precision, fn) in hooks.items():
        module = types.SimpleNamespace() if fn is None else types.SimpleNamespace(quantize_activations=fn)
        got = scale_guard.check(module, cases, precision)
        want = meta["checks"][name]
        assert set(got) == set(want), (name, sorted(got), sorted(want))
        same_outliers(got.pop("outliers"), want["outliers"], name)
        want = {k: v for k, v in want.items() if k != "outliers"}
        assert json.loads(json.dumps(got)) == want, (name, got, want)
