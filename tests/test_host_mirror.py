"""Host-side logic of the toolkit mirror that needs no GPU: the scale guard's stress inputs
equal the reference's bit for bit (golden), the format detection, the guard's early exits,
and CPU tensors refused by the GPU entry points."""

from __future__ import annotations

import types

import numpy as np
import pytest
import torch

from helpers import np_bf16_bits


@pytest.fixture(scope="module")
def kq():
    from kernel_agent_b200.kernels import quant

    return quant


def test_stress_inputs_match_the_reference(kq, golden):
    assert np.array_equal(np_bf16_bits(kq.mxfp8_stress_input((64, 256), seed=3)), golden["stress_mx"])
    assert np.array_equal(np_bf16_bits(kq.fp4_stress_input((64, 256), "nvfp4", seed=4)), golden["stress_fp4"])
    assert np.array_equal(np_bf16_bits(kq.fp4_stress_input((64, 256), "mxfp4", seed=5)), golden["stress_mx4"])
    with pytest.raises(ValueError, match="multiple of the MXFP8 block"):
        kq.mxfp8_stress_input((4, 48))
    with pytest.raises(ValueError, match="unknown FP4 format"):
        kq.fp4_stress_input((4, 64), "fp4")


def test_fp4_format_of(kq):
    assert kq.fp4_format_of(64, torch.zeros(2, 4, dtype=torch.float8_e4m3fn)) == "nvfp4"
    assert kq.fp4_format_of(64, torch.zeros(2, 2, dtype=torch.float8_e8m0fnu)) == "mxfp4"
    assert kq.fp4_format_of(64, torch.zeros(2, 4, dtype=torch.uint8)) == "nvfp4"
    assert kq.fp4_format_of(64, torch.zeros(2, 2, dtype=torch.uint8)) == "mxfp4"
    with pytest.raises(ValueError, match="unswizzled"):
        kq.fp4_format_of(64, torch.zeros(512, dtype=torch.uint8))


def test_scale_guard_unchecked_paths():
    from kernel_agent_b200.kernels import scale_guard

    x = torch.randn(4, 64)
    tie = torch.randn(2, 32)
    cases = [{"count": 3, "args": (x,)}, {"count": 1, "args": (torch.randn(2, 32),)}]
    assert scale_guard.activation(cases, 32) is x
    # equal counts keep the cases' order; keyword arguments come after positional ones
    assert scale_guard.activation([{"count": 2, "args": (5, tie)}, {"count": 2, "args": (x,)}], 32) is tie
    assert scale_guard.activation([{"args": (), "kwargs": {"x": x}}], 32) is x
    assert scale_guard.activation([{"args": (torch.randn(3, 5),)}], 32) is None
    assert scale_guard.activation([{"args": (torch.zeros(0, 32),)}], 32) is None
    # no quantisable input: neither outliers nor a check, only the note
    none = [{"count": 1, "args": (torch.randn(3, 5),)}]
    report = scale_guard.check(types.SimpleNamespace(), none, "fp8_mx")
    assert report["ok"] and not report["checked"] and "quantize_activations" in report["note"]
    assert "outliers" not in report
    fake = types.SimpleNamespace(quantize_activations=lambda t: (t, t))
    report = scale_guard.check(fake, none, "fp4_w4a4")
    assert report["ok"] and not report["checked"] and "nothing to quantise" in report["note"]
    # the outlier statistics are a GPU reduction: a CPU tensor is refused, not computed on the CPU
    with pytest.raises(ValueError, match="CUDA tensor required"):
        scale_guard.outliers(x)


def test_cpu_tensors_are_refused_by_the_checks(kq):
    x = torch.randn(4, 64)
    with pytest.raises(ValueError, match="CUDA tensor required"):
        kq.mxfp8_saturation(x, torch.zeros(4, 2, dtype=torch.uint8))
    with pytest.raises(ValueError, match="CUDA tensor required"):
        kq.fp4_scale_check(x, torch.zeros(4, 4, dtype=torch.float8_e4m3fn))
