"""The oracle's restatement of the reference's error reports against the reference's own
reports on seeded inputs (``tests/golden/make_golden_reports.py``), no GPU.

Strings, counts and byte sizes must be equal; the floats, which the reference reduces in fp32
in torch's order and rounds to 4 significant digits (6 for cosines), within about one unit
of the last printed digit.
"""

from __future__ import annotations

import json

import numpy as np
import pytest

from conftest import GOLDEN
from oracle import reports as orep
from oracle.formats import bf16_to_f32

TOL = {"output_cosine": (0.0, 3e-6), "output_gain": (0.0, 2e-5), "output_norm_ratio": (0.0, 2e-5)}


@pytest.fixture(scope="module")
def rg():
    with np.load(GOLDEN / "reports_golden.npz") as z:
        return {k: z[k] for k in z.files}


@pytest.fixture(scope="module")
def rmeta():
    return json.loads((GOLDEN / "reports_golden.json").read_text())


def close_reports(got: dict, want: dict, path: str = "") -> None:
    assert set(got) == set(want), (path, sorted(set(got) ^ set(want)))
    for key, w in want.items():
        g = got[key]
        where = f"{path}{key}"
        if isinstance(w, dict):
            close_reports(g, w, where + ".")
        elif isinstance(w, (str, bool)) or (isinstance(w, int) and not isinstance(w, bool) and key != "share"):
            assert g == w, (where, g, w)
        else:
            rel, ab = TOL.get(key, (2.5e-3, 1e-9))
            assert g == pytest.approx(w, rel=rel, abs=ab), (where, g, w)


def inputs(rg):
    return bf16_to_f32(rg["w128"]), bf16_to_f32(rg["w48"]), bf16_to_f32(rg["x"])


def test_weight_reports(rg, rmeta):
    w, w48, x = inputs(rg)
    close_reports(orep.fp8_error(w, 2), rmeta["fp8_error"])
    close_reports(orep.fp8_error(w, 2, x), rmeta["fp8_error_x"])
    close_reports(orep.int8_error(w, 2), rmeta["int8_error"])
    close_reports(orep.int8_error(w48, 2, x), rmeta["int8_error_x"])
    close_reports(orep.fp4_error(w, 2, "nvfp4", x)[0], rmeta["fp4_error_nv_x"])
    close_reports(orep.fp4_error(w48, 2, "mxfp4")[0], rmeta["fp4_error_mx"])
    close_reports(orep.fp4_error(w, 2, "nvfp4", unbiased=True)[0], rmeta["fp4_error_unbiased"])
    close_reports(orep.mxfp8_error(w, 2), rmeta["mxfp8_error"])


def test_layer_reports(rg, rmeta):
    w, w48, x = inputs(rg)
    close_reports(orep.mxfp8_error(w, 2, x), rmeta["mxfp8_error_x"])
    close_reports(orep.mxfp8_error(w48, 2, x), rmeta["mxfp8_error_x48"])
    close_reports(orep.fp8_w8a8_error(w, 2, x), rmeta["fp8_w8a8_error"])
    close_reports(orep.int8_w8a8_error(w, 2, x), rmeta["int8_w8a8_error"])
    s = orep.smoothquant_factors(np.abs(x).max(axis=0), w, 0.4)
    assert np.allclose(s, rg["smooth"], rtol=2e-6)
    close_reports(orep.int8_w8a8_error(w, 2, x, smooth=rg["smooth"]), rmeta["int8_w8a8_error_smooth"])


@pytest.mark.parametrize("case,kw", [
    ("fp4_w4a4_error", {}),
    ("fp4_w4a4_error_tensor", {"granularity": "tensor"}),
    ("fp4_w4a4_error_rot", {"rotate": 32}),
    ("fp4_w4a4_error_unbiased", {"unbiased": True}),
    ("fp4_w4a4_error_mx", {"fmt": "mxfp4"}),
])
def test_w4a4_reports(rg, rmeta, case, kw):
    w, _, x = inputs(rg)
    close_reports(orep.fp4_w4a4_error(w, x, **kw), rmeta[case])


def test_fp4_saturation(rg, rmeta):
    from oracle import quant as oq

    stress = bf16_to_f32(rg["stress"])
    _, xs, outer = oq.quantize_fp4_activations(stress, "nvfp4")
    assert orep.fp4_saturation(stress, xs, outer) == rmeta["fp4_saturation"]
    x = bf16_to_f32(rg["x"])
    _, xs, outer = oq.quantize_fp4_activations(x, "nvfp4")
    assert orep.fp4_saturation(x, xs, outer) == rmeta["fp4_saturation_plain"]
