"""The drop-in's Python boundary against the reference's own (``tests/golden/api.json``,
recorded from the reference by ``make_api.py``): every public function of
``kernel_agent.kernels.{quant,compare,scale_guard,kv_quant}`` exists in the mirror with the same
parameters (names, kinds, defaults: what a caller binds), and every public UPPER_CASE constant
``integrity.Snapshot`` freezes has the same value. Runs on the CPU (nothing is called)."""

from __future__ import annotations

import importlib
import json
import sys

import pytest

from conftest import GOLDEN

sys.path.insert(0, str(GOLDEN))
from make_api import MODULES, describe  # noqa: E402

API = json.loads((GOLDEN / "api.json").read_text())


@pytest.mark.parametrize("module", MODULES)
def test_functions_bind_like_the_reference(module):
    mine = describe(importlib.import_module(f"kernel_agent_b200.kernels.{module}"))["functions"]
    for name, params in API[module]["functions"].items():
        assert name in mine, f"{module}.{name} is missing"
        assert mine[name] == params, (f"{module}.{name}", mine[name], params)


@pytest.mark.parametrize("module", MODULES)
def test_constants_have_the_reference_values(module):
    mine = describe(importlib.import_module(f"kernel_agent_b200.kernels.{module}"))["constants"]
    for name, value in API[module]["constants"].items():
        assert name in mine, f"{module}.{name} is missing"
        assert mine[name] == value, (f"{module}.{name}", mine[name], value)
