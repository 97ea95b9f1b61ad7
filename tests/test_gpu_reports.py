"""The GPU error reports (``kernels/quant.py``: ``fp8_error``, ``int8_error``, ``fp4_error``,
``mxfp8_error``, ``fp8_w8a8_error``, ``int8_w8a8_error``, ``fp4_w4a4_error``,
``fp4_saturation``, ``smoothquant_factors``, ``fp4_w4a4_sensitivity``; ``kv_quant.fp8_kv_error``)
against the reference's own reports on the same inputs (``tests/golden/reports_golden.json``)
and the one-pass row sums (``kab_row_pair_stats``) against float64 numpy.

Strings, counts and sizes equal; weight fields within about one unit of the reports' last
digit (float64 sums against the reference's fp32 ones); output and activation fields within
the accumulation-order difference of the tcgen05 GEMMs against the reference's fp32 / float64
products.
"""

from __future__ import annotations

import json

import numpy as np
import pytest
import torch

from conftest import GOLDEN
from helpers import bits_to_bf16

pytestmark = pytest.mark.gpu
DEV = "cuda"
TOL = {"output_cosine": (0.0, 5e-6), "output_gain": (0.0, 5e-5), "output_norm_ratio": (0.0, 5e-5),
       "output_rel_l2": (1e-2, 1e-9), "activation_rel_l2": (5e-3, 1e-9)}


@pytest.fixture(scope="module")
def q():
    from kernel_agent_b200.kernels import quant

    return quant


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
        elif isinstance(w, str) or (isinstance(w, int) and key != "share"):
            assert g == w, (where, g, w)
        else:
            rel, ab = TOL.get(key, (2.5e-3, 1e-9))
            assert g == pytest.approx(w, rel=rel, abs=ab), (where, g, w)


def test_pair_stats_against_numpy(q):
    g = torch.Generator().manual_seed(5)
    x = torch.randn(37, 1000, generator=g)
    y = x + 0.01 * torch.randn(37, 1000, generator=g)
    x[3, :10] = 0.0
    y[3, :5] = 0.0
    y[4] = 0.0
    for dx, dy in ((torch.float32, torch.float32), (torch.bfloat16, torch.float32), (torch.float16, torch.bfloat16)):
        xa, ya = x.to(dx), y.to(dy)
        st = q._pair_stats(xa.to(DEV), ya.to(DEV)).cpu().numpy()
        a, b = xa.double().numpy(), ya.double().numpy()
        want = np.stack([(a * a).sum(1), (b * b).sum(1), ((a - b) ** 2).sum(1), (a * b).sum(1), np.abs(a).max(1),
                         (a != 0).sum(1), ((a != 0) & (b == 0)).sum(1), np.abs(b).max(1)], axis=1)
        assert np.allclose(st, want, rtol=1e-12, atol=0), (dx, dy)
    # NaN propagates into the sums and the maximum
    x[7, 3] = float("nan")
    st = q._pair_stats(x.to(DEV), y.to(DEV)).cpu().numpy()
    assert np.isnan(st[7, 0]) and np.isnan(st[7, 4]) and np.isfinite(st[6]).all()


def test_weight_reports(q, rg, rmeta):
    w, w48, x = (bits_to_bf16(rg[k]) for k in ("w128", "w48", "x"))
    close_reports(q.fp8_error(w, *q.quantize_fp8(w)), rmeta["fp8_error"])
    close_reports(q.fp8_error(w, *q.quantize_fp8(w), x), rmeta["fp8_error_x"])
    close_reports(q.int8_error(w, *q.quantize_int8(w)), rmeta["int8_error"])
    close_reports(q.int8_error(w48, *q.quantize_int8(w48), x), rmeta["int8_error_x"])
    close_reports(q.fp4_error(w, *q.quantize_fp4(w, "nvfp4"), x), rmeta["fp4_error_nv_x"])
    close_reports(q.fp4_error(w48, *q.quantize_fp4(w48, "mxfp4")), rmeta["fp4_error_mx"])
    close_reports(q.fp4_error(w, *q.quantize_fp4(w, "nvfp4", unbiased=True)), rmeta["fp4_error_unbiased"])
    close_reports(q.mxfp8_error(w, *q.quantize_mxfp8(w)), rmeta["mxfp8_error"])


def test_layer_reports(q, rg, rmeta):
    w, w48, x = (bits_to_bf16(rg[k]) for k in ("w128", "w48", "x"))
    close_reports(q.mxfp8_error(w, *q.quantize_mxfp8(w), x), rmeta["mxfp8_error_x"])
    close_reports(q.mxfp8_error(w48, *q.quantize_mxfp8(w48), x), rmeta["mxfp8_error_x48"])
    close_reports(q.fp8_w8a8_error(w, *q.quantize_fp8(w), x), rmeta["fp8_w8a8_error"])
    close_reports(q.int8_w8a8_error(w, *q.quantize_int8(w), x), rmeta["int8_w8a8_error"])
    s = q.smoothquant_factors(x.float().abs().amax(dim=0), w, 0.4)
    assert torch.allclose(s.cpu(), torch.from_numpy(rg["smooth"]), rtol=2e-6)
    sm = torch.from_numpy(rg["smooth"]).to(DEV)
    close_reports(q.int8_w8a8_error(w, *q.quantize_int8(w, sm), x, smooth=sm), rmeta["int8_w8a8_error_smooth"])


@pytest.mark.parametrize("case,kw", [
    ("fp4_w4a4_error", {}),
    ("fp4_w4a4_error_tensor", {"granularity": "tensor"}),
    ("fp4_w4a4_error_rot", {"rotate": 32}),
    ("fp4_w4a4_error_unbiased", {"unbiased": True}),
    ("fp4_w4a4_error_mx", {"fmt": "mxfp4"}),
])
def test_w4a4_reports(q, rg, rmeta, case, kw):
    w, x = bits_to_bf16(rg["w128"]), bits_to_bf16(rg["x"])
    fmt = kw.get("fmt", "nvfp4")
    wq = q.hadamard_rotate(w.float(), kw["rotate"]) if "rotate" in kw else w
    codes = q.quantize_fp4(wq, fmt, unbiased=kw.get("unbiased", False))
    close_reports(q.fp4_w4a4_error(w, *codes, x, **kw), rmeta[case])


def test_fp4_saturation(q, rg, rmeta):
    stress = bits_to_bf16(rg["stress"])
    _, xs, outer = q.quantize_fp4_activations(stress, "nvfp4")
    assert q.fp4_saturation(stress, xs, outer) == rmeta["fp4_saturation"]
    x = bits_to_bf16(rg["x"])
    _, xs, outer = q.quantize_fp4_activations(x, "nvfp4")
    assert q.fp4_saturation(x, xs, outer) == rmeta["fp4_saturation_plain"]


def test_sensitivity_probe(q):
    torch.manual_seed(0)

    class Block(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.a = torch.nn.Linear(256, 512, bias=False)
            self.b = torch.nn.Linear(256, 512, bias=False)  # reads the same inputs as a
            self.c = torch.nn.Linear(512, 256, bias=False)

        def forward(self, x):
            return self.c(torch.relu(self.a(x)) * self.b(x))

    m = Block().to(DEV).to(torch.bfloat16)
    xs = [torch.randn(48, 256, device=DEV, dtype=torch.bfloat16) for _ in range(3)]
    rows = q.fp4_w4a4_sensitivity(m, lambda: [m(x) for x in xs], calls=2)
    assert [r["name"] for r in rows] and {r["name"] for r in rows} == {"a", "b", "c"}
    assert all(rows[i]["w4a4_rel_l2"] >= rows[i + 1]["w4a4_rel_l2"] for i in range(len(rows) - 1))
    by = {r["name"]: r for r in rows}
    assert by["b"]["input_group"] == "a" and by["c"]["input_group"] == "c" and by["a"]["rows"] == 96
    assert sum(r["flop_share"] for r in rows) == pytest.approx(1.0, abs=2e-3)
    assert all(r["fp8_rel_l2"] < r["w4a4_rel_l2"] for r in rows)
