"""The comparator's routing on the GPU (grown caches, rows written into an input, in-place
updates, nested structures; the difference census ``kab_diff_census`` underneath) against
the reference's own results on the same tensors (``tests/golden/routing_golden.*``, made by
``make_golden_routing.py``): verdicts, the parts judged, counts of changed elements, mismatch
fractions and worst ratios equal; cosine / relative L2 / norm ratios within the reference's
fp32 reduction noise; error texts equal up to those numbers."""

from __future__ import annotations

import json
import re

import numpy as np
import pytest
import torch

from conftest import GOLDEN

pytestmark = pytest.mark.gpu
DEV = "cuda"
EXACT = ("ok", "grown", "written", "kept_changed", "changed_elements", "mismatch_frac", "max_err_ratio",
         "max_abs_err", "tier", "atol", "rtol", "name")
CLOSE = {"cosine": 2e-5, "rel_l2": 2e-4, "norm_ratio": 2e-5, "element_ratio": 2e-4, "max_err_over_rms": 2e-4,
         "mean_abs_err": 1e-5, "rounding_spread": 2e-5, "error_over_spread": 2e-3}


@pytest.fixture(scope="module")
def routing():
    meta = json.loads((GOLDEN / "routing_golden.json").read_text())
    tensors = {}
    with np.load(GOLDEN / "routing_golden.npz") as z:
        for name in z.files:
            dtype = getattr(torch, meta["dtypes"][name])
            arr = z[name]
            if dtype in (torch.bfloat16, torch.float16):
                t = torch.from_numpy(arr.view(np.int16)).view(dtype)
            else:
                t = torch.from_numpy(arr)
            tensors[name] = t.to(DEV)
    return tensors, meta["cases"]


def shape_of(error):
    return None if error is None else re.sub(r"[-+]?\d+(\.\d+)?(e[-+]?\d+)?%?", "#", error)


def agree(got: dict, want: dict, label) -> None:
    assert set(got) == set(want), (label, sorted(got), sorted(want))
    for key in EXACT:
        if key in want:
            assert got[key] == want[key], (label, key, got[key], want[key])
    for key, tol in CLOSE.items():
        if key in want:
            assert abs(got[key] - want[key]) <= tol * max(1.0, abs(want[key])), (label, key, got[key], want[key])
    assert shape_of(got.get("error")) == shape_of(want.get("error")), (label, got.get("error"), want.get("error"))


def test_routing_matches_the_reference(routing):
    from kernel_agent_b200.kernels import compare

    t, cases = routing

    def resolve(v):
        if isinstance(v, str):
            return t[v]
        if isinstance(v, list):
            return [resolve(x) for x in v]
        if isinstance(v, dict):
            return {k: resolve(x) for k, x in v.items()}
        return v

    for i, case in enumerate(cases):
        fn, kw, want = case["fn"], case.get("kw", {}), case["result"]
        label = (i, fn, case.get("new"))
        if fn == "output":
            agree(compare.compare_output("y", resolve(case["ref"]), resolve(case["new"]), resolve(case["inputs"]), **kw),
                  want, label)
        elif fn == "grown":
            agree(compare.compare_grown("y", resolve(case["before"]), resolve(case["ref"]), resolve(case["new"]),
                                        case["dim"], **kw), want, label)
        elif fn == "structures":
            got = compare.compare_structures(resolve(case["ref"]), resolve(case["new"]), inputs=resolve(case["inputs"]),
                                             **kw)
            assert len(got) == len(want), label
            for g, w in zip(got, want):
                agree(g, w, label + (w["name"],))
        elif fn == "side_effects":
            got = compare.compare_side_effects_flat(resolve(case["pre"]), resolve(case["ref"]), resolve(case["new"]),
                                                    **kw)
            assert len(got) == len(want), label
            for g, w in zip(got, want):
                agree(g, w, label + (w["name"],))
        elif fn == "written_box":
            box = compare.written_box(resolve(case["before"]), resolve(case["after"]))
            assert (None if box is None else [b.tolist() for b in box]) == want, label
        else:
            assert compare.grown_dim(resolve(case["before"]), resolve(case["after"])) == want, label


def test_census_counts_and_hits():
    """The census itself on hand-made differences: NaN equal to NaN or not, a slice along one
    dimension, the union of two candidates, per-dimension hits and a box left out, float64
    and integer tensors."""
    from kernel_agent_b200.kernels import compare

    base = torch.randn(3, 5, 7, device=DEV)
    base[0, 0, 0] = float("nan")
    a = base.clone()
    a[1, 2, 3] += 1
    a[2, 4, 6] = -a[2, 4, 6] - 1
    assert compare._census(a, base).count == 2
    assert compare._census(a, base, nan_equal=False).count == 3  # NaN != NaN
    found = compare._census(a, base, hits=True, mask=True)
    assert [h.nonzero().flatten().tolist() for h in found.hits] == [[1, 2], [2, 4], [3, 6]]
    assert found.mask.shape == base.shape and int(found.mask.sum()) == 2 and bool(found.mask[1, 2, 3])
    box = [torch.tensor([False, True, False], device=DEV), torch.ones(5, dtype=torch.bool, device=DEV),
           torch.ones(7, dtype=torch.bool, device=DEV)]
    assert compare._census(a, base, outside=box).count == 1  # [1, 2, 3] is inside the box
    b = base.clone()
    b[0, 1, 1] += 2
    assert compare._census(a, base, also=b).count == 3
    grown = torch.cat([a, torch.randn(3, 2, 7, device=DEV)], dim=1)
    assert compare._census(grown, base, dim=1, length=5).count == 2  # the kept slice only
    assert compare._census(a.double(), base.double()).count == 2
    ints = torch.arange(40, device=DEV, dtype=torch.int64).reshape(8, 5)
    other = ints.clone()
    other[7, 4] = -1
    assert compare._census(other, ints).count == 1
    flags = torch.zeros(10, dtype=torch.bool, device=DEV)
    assert compare._census(flags.clone().fill_(True), flags).count == 10
    assert compare._census(torch.tensor(1.0, device=DEV), torch.tensor(2.0, device=DEV), mask=True).mask.shape == ()
