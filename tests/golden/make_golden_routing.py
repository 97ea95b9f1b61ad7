"""Generate the golden routing results that pin the GPU comparator's routing (grown caches,
rows written into an input, in-place updates, nested structures) to the reference's.

Run in a container where the reference sources are present (they are not on the GPU box):

    python tests/golden/make_golden_routing.py /path/to/kernel-agent/src

It imports the reference's own ``kernel_agent.kernels.compare``, runs ``compare_output``,
``compare_structures``, ``compare_side_effects_flat``, ``grown_dim`` and ``written_box`` on
seeded scenarios (CPU tensors) and writes ``routing_golden.npz`` (every tensor: 2-byte floats
as uint16 bits) and ``routing_golden.json`` (the scenarios, naming their tensors, and the
results). The fixtures are committed; the tests only read them.
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


def scenarios() -> tuple[dict[str, torch.Tensor], list[dict]]:
    g = torch.Generator().manual_seed(44)
    bf = torch.bfloat16
    t: dict[str, torch.Tensor] = {}
    cases: list[dict] = []

    def keep(name: str, x: torch.Tensor) -> str:
        t[name] = x
        return name

    # a KV cache grown by one token along dim 2
    before = keep("kv", torch.randn(1, 4, 64, 16, generator=g).to(bf))
    row = torch.randn(1, 4, 1, 16, generator=g).to(bf)
    grown = keep("kv_grown", torch.cat([t[before], row], dim=2))
    keep("kv_grown_close", (t[grown].float() * (1 + 0.001 * torch.randn(t[grown].shape, generator=g))).to(bf))
    drift = t[grown].clone()
    drift[0, 1, 5, 3] += 0.5
    keep("kv_grown_kept_drift", drift)
    wrong = t[grown].clone()
    wrong[0, :, 64, :] = torch.randn(4, 16, generator=g).to(bf)
    keep("kv_grown_new_wrong", wrong)
    for tier in ("exact", "near-lossless-kv"):
        for new in ("kv_grown", "kv_grown_close", "kv_grown_kept_drift", "kv_grown_new_wrong"):
            cases.append({"fn": "output", "ref": grown, "new": new, "inputs": [before], "kw": {"tier": tier}})
    # the reference also rescaled part of the kept rows (the changed-elements path)
    rescaled = t[grown].clone()
    rescaled[0, 2, :8, :] = (rescaled[0, 2, :8, :].float() * 1.5).to(bf)
    keep("kv_rescaled", rescaled)
    close = (rescaled.float() * (1 + 0.002 * torch.randn(rescaled.shape, generator=g))).to(bf)
    keep("kv_rescaled_close", close)
    off = rescaled.clone()
    off[0, 2, :8, :] = t[before][0, 2, :8, :]
    keep("kv_rescaled_missed", off)
    for new in ("kv_rescaled_close", "kv_rescaled_missed"):
        cases.append({"fn": "grown", "before": before, "ref": "kv_rescaled", "new": new, "dim": 2, "kw": {}})
    # grown along the channels (last dim), judged on redrawn inputs with per-channel floors
    base = keep("ch", torch.randn(32, 24, generator=g))
    ext = keep("ch_grown", torch.cat([t[base], torch.randn(32, 8, generator=g)], dim=1))
    keep("ch_grown_close", t[ext] + 0.01 * torch.randn(t[ext].shape, generator=g))
    cases.append({"fn": "output", "ref": ext, "new": "ch_grown_close", "inputs": [base],
                  "kw": {"tier": "near-lossless", "perturbed": True}})
    # rows written into a static cache (functional index_copy of one slot)
    static = keep("static", torch.randn(1, 4, 64, 16, generator=g).to(bf))
    t[static][0, 3, 40, 7] = float("nan")  # NaN equal to NaN where nothing is written
    written = t[static].clone()
    written[:, :, 10, :] = torch.randn(1, 4, 16, generator=g).to(bf)
    keep("static_written", written)
    keep("static_written_close", (written.float() * (1 + 0.001 * torch.randn(written.shape, generator=g))).to(bf))
    wrong_slot = t[static].clone()
    wrong_slot[:, :, 11, :] = written[:, :, 10, :]
    keep("static_wrong_slot", wrong_slot)
    for new in ("static_written", "static_written_close", "static_wrong_slot"):
        cases.append({"fn": "output", "ref": "static_written", "new": new, "inputs": ["static"], "kw": {}})
    # scattered changes are no written box: compared whole
    scattered = t[static].clone()
    flat = scattered.view(-1)
    idx = torch.randperm(flat.numel(), generator=g)[:40]
    flat[idx] = (flat[idx].float() + 1).to(bf)
    keep("static_scattered", scattered)
    cases.append({"fn": "output", "ref": "static_scattered", "new": "static_scattered", "inputs": ["static"], "kw": {}})
    cases.append({"fn": "written_box", "before": "static", "after": "static_written"})
    cases.append({"fn": "written_box", "before": "static", "after": "static_scattered"})
    cases.append({"fn": "grown_dim", "before": before, "after": grown})
    # in-place updates of arguments (IEEE != : a NaN element counts as changed)
    arg = keep("arg", torch.randn(8, 32, generator=g))
    arg_nan = t[arg].clone()
    arg_nan[1, 1] = float("nan")
    keep("arg_nan", arg_nan)
    upd = arg_nan.clone()
    upd[2, :4] += 1.0
    keep("arg_upd", upd)
    keep("arg_upd_close", upd + 1e-6 * (upd == upd) * torch.randn(upd.shape, generator=g))
    bad = upd.clone()
    bad[2, 0] += 0.5
    keep("arg_upd_bad", bad)
    count = keep("count", torch.tensor([5, 0, 7], dtype=torch.int32))
    keep("count_next", torch.tensor([6, 0, 7], dtype=torch.int32))
    keep("count_wrong", torch.tensor([6, 1, 7], dtype=torch.int32))
    for new in ("arg_upd", "arg_upd_close", "arg_upd_bad", "arg_nan"):
        cases.append({"fn": "side_effects", "pre": {"a": "arg_nan", "k": count, "c": before},
                      "ref": {"a": "arg_upd", "k": "count_next", "c": grown},
                      "new": {"a": new, "k": "count_wrong" if new == "arg_upd_bad" else "count_next",
                              "c": "kv_grown_kept_drift"}, "kw": {}})
    # nested structures: a missing output, a grown cache inside a dict
    cases.append({"fn": "structures", "ref": {"y": "ch_grown", "cache": grown, "extra": base},
                  "new": {"y": "ch_grown_close", "cache": "kv_grown_close"}, "inputs": [before],
                  "kw": {"tier": "near-lossless"}})
    return t, cases


def main(src: str) -> None:
    sys.path.insert(0, src)
    from kernel_agent.kernels import compare  # noqa: E402  (the reference)

    t, cases = scenarios()

    def resolve(v):
        if isinstance(v, str):
            return t[v]
        if isinstance(v, list):
            return [resolve(x) for x in v]
        if isinstance(v, dict):
            return {k: resolve(x) for k, x in v.items()}
        return v

    for case in cases:
        fn, kw = case["fn"], case.get("kw", {})
        if fn == "output":
            res = compare.compare_output("y", resolve(case["ref"]), resolve(case["new"]), resolve(case["inputs"]), **kw)
        elif fn == "grown":
            res = compare.compare_grown("y", resolve(case["before"]), resolve(case["ref"]), resolve(case["new"]),
                                        case["dim"], **kw)
        elif fn == "structures":
            res = compare.compare_structures(resolve(case["ref"]), resolve(case["new"]),
                                             inputs=resolve(case["inputs"]), **kw)
        elif fn == "side_effects":
            res = compare.compare_side_effects_flat(resolve(case["pre"]), resolve(case["ref"]),
                                                    resolve(case["new"]), **kw)
        elif fn == "written_box":
            box = compare.written_box(resolve(case["before"]), resolve(case["after"]))
            res = None if box is None else [b.tolist() for b in box]
        else:
            res = compare.grown_dim(resolve(case["before"]), resolve(case["after"]))
        case["result"] = res
    np.savez_compressed(HERE / "routing_golden.npz", **{k: bits(v) for k, v in t.items()})
    dtypes = {k: str(v.dtype).replace("torch.", "") for k, v in t.items()}
    (HERE / "routing_golden.json").write_text(json.dumps({"dtypes": dtypes, "cases": cases}, indent=1) + "\n")
    print(f"wrote {len(t)} tensors and {len(cases)} cases")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit(f"usage: python {sys.argv[0]} <path to the reference's src directory>")
    main(sys.argv[1])
