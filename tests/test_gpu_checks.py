"""The scale-rule checks on the GPU (one reduction each) against the reference's results on
its stress inputs (golden) and the oracle on random and edge-case inputs, exactly; the scale
guard's report for good and saturating quantisers."""

from __future__ import annotations

import types

import numpy as np
import pytest
import torch

from helpers import np_bytes, np_values
from oracle import quant as oq
from oracle.formats import bf16_to_f32

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(scope="module")
def kq():
    from kernel_agent_b200.kernels import quant

    return quant


def bf(g, key):
    return torch.from_numpy(g[key].view(np.int16)).view(torch.bfloat16)


def test_golden_checks(kq, golden, golden_meta):
    for chk in golden_meta["checks"]:
        x = bf(golden, chk["input"]).to(DEV)
        if chk["kind"] == "mxfp8":
            _, s = kq.quantize_mxfp8(x, chk["rule"])
            got = kq.mxfp8_saturation(x, s)
        else:
            fmt = chk["fmt"]
            _, s, o = kq.quantize_fp4_activations(x, fmt)
            if chk.get("variant") == "trunc":
                s = torch.from_numpy(golden["stress_fp4_trunc_scales"]).view(torch.float8_e4m3fn).to(DEV)
            got = kq.fp4_scale_check(x, s, o, fmt)
        assert got == chk["result"], (chk, got)


@pytest.mark.parametrize("seed", [0, 1])
def test_checks_against_oracle(kq, seed):
    g = torch.Generator().manual_seed(seed)
    x = (torch.randn(96, 512, generator=g) * torch.logspace(-20, 20, 96)[:, None]).to(torch.bfloat16)
    x[3] = 0
    x[5, 17] = float("nan")
    x[6, 40] = float("inf")
    xd = x.to(DEV)
    xn = np_values(x)
    # MXFP8: the ceil rule, the floor rule, and arbitrary (not power-of-two) scale values
    for rule in ("ceil", "floor"):
        _, s = kq.quantize_mxfp8(xd, rule)
        assert kq.mxfp8_saturation(xd, s) == oq.mxfp8_saturation(xn, np_bytes(s)), rule
    vals = torch.rand(96, 16, generator=g) * 4
    vals[0, 0] = 0
    assert kq.mxfp8_saturation(xd, vals.to(DEV)) == oq.mxfp8_saturation(xn, vals.numpy())
    # NVFP4 / MXFP4 with their own outer scales, scaled-down scales and odd outers
    for fmt in ("nvfp4", "mxfp4"):
        _, s, o = kq.quantize_fp4_activations(xd, fmt)
        sb = np_bytes(s)
        assert kq.fp4_scale_check(xd, s, o, fmt) == oq.fp4_scale_check(xn, sb, o.cpu().numpy(), fmt), fmt
        o2 = o.clone()
        o2[1] = 0.0
        o2[2] = float("inf")
        assert kq.fp4_scale_check(xd, s, o2, fmt) == oq.fp4_scale_check(xn, sb, o2.cpu().numpy(), fmt), fmt
        assert kq.fp4_scale_check(xd, s, None, fmt) == oq.fp4_scale_check(xn, sb, None, fmt), fmt


def test_scale_guard_reports(kq):
    from kernel_agent_b200.kernels import scale_guard

    x = torch.randn(64, 256, device=DEV).to(torch.bfloat16)
    cases = [{"count": 1, "args": (x,)}]
    good = types.SimpleNamespace(quantize_activations=lambda t: kq.quantize_mxfp8(t, "ceil"))
    report = scale_guard.check(good, cases, "fp8_mx")
    assert report["ok"] and report["checked"] and report["stress"]["saturated"] == 0
    floor = types.SimpleNamespace(quantize_activations=lambda t: kq.quantize_mxfp8(t, "floor"))
    report = scale_guard.check(floor, cases, "fp8_mx")
    assert not report["ok"] and "saturate" in report["error"]
    fp4 = types.SimpleNamespace(quantize_activations=lambda t: kq.quantize_fp4_activations(t, "nvfp4"))
    report = scale_guard.check(fp4, cases, "fp4_w4a4")
    assert report["ok"] and report["stress"]["format"] == "nvfp4"

    def truncating(t):
        c, s, o = kq.quantize_fp4_activations(t, "nvfp4")
        return c, (torch.floor(s.float() * 8) / 8).to(torch.float8_e4m3fn), o

    report = scale_guard.check(types.SimpleNamespace(quantize_activations=truncating), cases, "fp4_w4a4")
    assert not report["ok"] and report["input"] == "stress" and "round the block scale" in report["error"]
