"""Record the reference's public Python interface for the drop-in check (``tests/test_api.py``).

Run in a container where the reference sources are present (they are not on the GPU box):

    python tests/golden/make_api.py /path/to/kernel-agent/src

For each module the drop-in replaces (``kernel_agent.kernels.{quant,compare,scale_guard,
kv_quant}``) it writes to ``api.json``: every public function defined there (name, and per
parameter its name, kind and default: what a caller binds; annotations are not part of the
contract) and every public UPPER_CASE constant with a plain value (what
``kernel_agent.kernels.integrity.Snapshot`` freezes by value), serialised by :func:`plain`.
The fixture is committed; the test only reads it.
"""

from __future__ import annotations

import importlib
import inspect
import json
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
MODULES = ("quant", "compare", "scale_guard", "kv_quant")


def plain(value):
    """A JSON form of a constant: numbers, strings and booleans as they are, torch dtypes as
    their names, containers element by element (dict keys as strings), anything else None."""
    import torch

    if isinstance(value, bool | int | float | str) or value is None:
        return value
    if isinstance(value, torch.dtype):
        return f"torch.{str(value).split('.')[-1]}"
    if isinstance(value, tuple | list):
        return [plain(v) for v in value]
    if isinstance(value, frozenset | set):
        return sorted(plain(v) for v in value)
    if isinstance(value, dict):
        return {str(plain(k)): plain(v) for k, v in value.items()}
    return None


def parameters(fn) -> list:
    out = []
    for p in inspect.signature(fn).parameters.values():
        default = None if p.default is inspect.Parameter.empty else repr(p.default)
        out.append([p.name, p.kind.name, default])
    return out


def describe(module) -> dict:
    functions, constants = {}, {}
    for name, value in vars(module).items():
        if name.startswith("_"):
            continue
        if inspect.isfunction(value) and value.__module__ == module.__name__:
            functions[name] = parameters(value)
        elif name.isupper() and not callable(value):
            frozen = plain(value)
            if frozen is not None:
                constants[name] = frozen
    return {"functions": functions, "constants": constants}


def main(src: str) -> None:
    sys.path.insert(0, src)
    api = {m: describe(importlib.import_module(f"kernel_agent.kernels.{m}")) for m in MODULES}
    (HERE / "api.json").write_text(json.dumps(api, indent=1, sort_keys=True) + "\n")
    print({m: (len(v["functions"]), len(v["constants"])) for m, v in api.items()})


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit(f"usage: python {sys.argv[0]} <path to the reference's src directory>")
    main(sys.argv[1])
