"""The GPU comparator against the reference's own results (golden) and the oracle: verdicts,
the problems named, mismatch fractions and outlier ratios bit for bit; cosine, relative L2
and the norm / element ratios within the reference's fp32 reduction noise."""

from __future__ import annotations

import re

import numpy as np
import pytest
import torch

from helpers import np_values
from oracle import compare as ocmp

pytestmark = pytest.mark.gpu
DEV = "cuda"
TORCH = {"bfloat16": torch.bfloat16, "float16": torch.float16, "float32": torch.float32}


@pytest.fixture(scope="module")
def kc():
    from kernel_agent_b200.kernels import compare

    return compare


def shape_of(error):
    return None if error is None else re.sub(r"[-+]?\d+(\.\d+)?(e[-+]?\d+)?", "#", error)


def agree(got, want, label):
    assert got["ok"] == want["ok"], (label, got, want)
    assert shape_of(got.get("error")) == shape_of(want.get("error")), (label, got, want)
    for key in ("mismatch_frac", "max_err_ratio", "max_abs_err"):
        assert got.get(key) == want.get(key), (label, key, got.get(key), want.get(key))
    for key, tol in (("cosine", 2e-5), ("rel_l2", 2e-4), ("norm_ratio", 2e-5), ("element_ratio", 2e-4),
                     ("max_err_over_rms", 2e-4), ("mean_abs_err", 1e-5), ("rounding_spread", 2e-5),
                     ("error_over_spread", 2e-3)):
        if key in want:
            assert abs(got[key] - want[key]) <= tol * max(1.0, abs(want[key])), (label, key, got[key], want[key])


def tensor_of(golden, key, dtype):
    arr = golden[key]
    if dtype == "bfloat16":
        return torch.from_numpy(arr.view(np.int16)).view(torch.bfloat16).to(DEV)
    return torch.from_numpy(arr).to(DEV)


def test_golden_cases(kc, golden, golden_meta):
    for case in golden_meta["compare"]:
        dt = case["dtype"]
        ref, new = tensor_of(golden, case["ref"], dt), tensor_of(golden, case["new"], dt)
        rer = None if case["rer"] is None else tensor_of(golden, case["rer"], dt)
        got = kc.compare_tensors(case["result"]["name"], ref, new, rerounded=rer, **case["kw"])
        agree(got, case["result"], case["result"]["name"])


@pytest.mark.parametrize("tier", ["exact", "near-lossless", "relaxed-fp4a"])
@pytest.mark.parametrize("perturbed", [False, True])
def test_random_against_oracle(kc, tier, perturbed):
    g = torch.Generator().manual_seed(3)
    for shape, noise in (((257, 300), 0.01), ((64, 4096), 0.05), ((4096,), 0.002), ((3, 17, 64), 0.3)):
        ref = torch.randn(*shape, generator=g).to(torch.bfloat16)
        new = (ref.float() + noise * torch.randn(*shape, generator=g)).to(torch.bfloat16)
        got = kc.compare_tensors("x", ref.to(DEV), new.to(DEV), tier=tier, perturbed=perturbed)
        want = ocmp.compare_tensors("x", np_values(ref), np_values(new), "bf16", tier=tier, perturbed=perturbed)
        agree(got, want, (shape, tier, perturbed))


def test_nonfinite_and_integers(kc):
    a = torch.randn(2000).to(torch.bfloat16)
    a[3], a[9] = float("nan"), float("inf")
    b = a.clone()
    b[5] += 1
    got = kc.compare_tensors("x", a.to(DEV), b.to(DEV))
    agree(got, ocmp.compare_tensors("x", np_values(a), np_values(b), "bf16"), "nonfinite")
    c = b.clone()
    c[9] = -float("inf")
    got = kc.compare_tensors("x", a.to(DEV), c.to(DEV))
    assert not got["ok"] and "+inf at 1 positions" in got["error"] and "-inf" in got["error"]
    i = torch.arange(100, device=DEV)
    assert kc.compare_tensors("i", i, i.clone())["ok"]
    res = kc.compare_tensors("i", i, i + (i == 7))
    assert not res["ok"] and res["mismatch_frac"] == float(np.float32(1) / np.float32(100))


def test_structures_caches_and_errors(kc):
    ref = (torch.ones(2, device=DEV), torch.ones(3, device=DEV))
    res = kc.compare_structures(ref, (torch.ones(2, device=DEV),))
    assert [r["ok"] for r in res] == [True, False]
    before = torch.randn(1, 4, 64, 16, device=DEV).to(torch.bfloat16)
    new_row = torch.randn(1, 4, 1, 16, device=DEV).to(torch.bfloat16)
    grown = torch.cat([before, new_row], dim=2)
    res = kc.compare_output("cache", grown, grown.clone(), (before,))
    assert res["ok"] and res["grown"] == {"dim": 2, "kept": 64, "appended": 1}
    bad = grown.clone()
    bad[0, 0, 0, 0] += 1
    assert not kc.compare_output("cache", grown, bad, (before,))["ok"]
    assert "shape" in kc.compare_tensors("x", torch.zeros(4, device=DEV), torch.zeros(5, device=DEV))["error"]
    with pytest.raises(ValueError, match="CUDA tensor required"):
        kc.compare_tensors("x", torch.zeros(4), torch.zeros(4))


def test_full_size_output_verdict_is_stable(kc):
    """A config-4-sized bf16 output: the verdict and its counts do not change between calls
    (the reduction is deterministic: per-block partials added in index order)."""
    g = torch.Generator(device=DEV).manual_seed(0)
    ref = torch.randn(8192, 28672, generator=g, device=DEV).to(torch.bfloat16)
    new = (ref.float() * (1 + 0.01 * torch.randn(8192, 28672, generator=g, device=DEV))).to(torch.bfloat16)
    a = kc.compare_tensors("y", ref, new, tier="near-lossless-fp4a")
    b = kc.compare_tensors("y", ref, new, tier="near-lossless-fp4a")
    assert a == b and a["ok"]
    sub = slice(0, 64)
    want = ocmp.compare_tensors("y", np_values(ref[sub]), np_values(new[sub]), "bf16", tier="near-lossless-fp4a")
    got = kc.compare_tensors("y", ref[sub], new[sub], tier="near-lossless-fp4a")
    agree(got, want, "row sample")
