"""What a b200 build writes for one module, and how it is written.

For module `m` the build writes, into the output directory:

* `m.cu`   -- the generated CUDA C++ (kernels, host wrappers, exported entry points);
* `m.so`   -- that source compiled for sm_100a;
* `m.json` -- the manifest the runtime loads: every exported function with its
  parameters (kind, element type, role) and its kernels.

Only this module and `translate` touch PPy's IR; the manifest is all the runtime needs.
"""

from __future__ import annotations

import json
from pathlib import Path

from . import codegen
from . import plan as P
from .toolchain import ARCH, build_module

MANIFEST_FORMAT = "ppy-b200/1"


def plan_and_source(module) -> tuple[P.ModulePlan, str]:
    from .translate import plan_module

    planned = plan_module(module)
    source = codegen.module_source(planned, planned.device_sources, planned.parallel_kernels)
    return planned, source


def manifest(planned: P.ModulePlan) -> dict:
    functions = []
    for fn in planned.functions:
        entry = {
            "name": fn.name,
            "symbol": fn.symbol,
            "kind": fn.kind,
            "result": fn.result,
            "params": [
                {"name": p.name, "kind": p.kind, "dtype": p.dtype, "role": p.role}
                for p in fn.params
            ],
            "kernels": [k.kind for k in fn.kernels],
        }
        functions.append(entry)
    return {
        "format": MANIFEST_FORMAT,
        "arch": ARCH,
        "module": planned.name,
        "source": f"{planned.name}.cu",
        "library": f"{planned.name}.so",
        "functions": functions,
        "notes": list(planned.notes),
    }


def write_module(module, output: Path, compile_library: bool = True) -> list[Path]:
    """Plan, generate and (optionally) compile one module into `output`."""
    planned, source = plan_and_source(module)
    output.mkdir(parents=True, exist_ok=True)
    cu = output / f"{planned.name}.cu"
    cu.write_text(source, encoding="utf-8")
    meta = output / f"{planned.name}.json"
    meta.write_text(json.dumps(manifest(planned), indent=1) + "\n", encoding="utf-8")
    written = [cu, meta]
    if compile_library:
        written.append(build_module(cu, output / f"{planned.name}.so"))
    return written
