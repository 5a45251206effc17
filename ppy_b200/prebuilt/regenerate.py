"""Regenerate the prebuilt modules from the IR fixtures in tests/golden/.

Each `tests/golden/<name>.ppyir` is canonical IR as PPy's shared passes hand it to a
backend; this runs the b200 backend's translation on it -- the same code
`ppy build <name>.ppyir --backend b200` runs -- and writes `<name>/<name>.cu` and
`<name>/<name>.json` here. The libraries (`<name>.so`) are compiled from those by
`__graft_entry__.build()` or on first load. Needs PPy's compiler importable
(`--reference /path/to/PPy`).
"""

from __future__ import annotations

import argparse
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
GOLDEN = REPO / "tests" / "golden"
MODULES = ("gelu", "rows", "chain", "reductions", "collatz", "matmul", "matmul_bf16",
           "matmul_bf16_8192", "gpt2_layernorm")


def regenerate(names=MODULES, compile_library: bool = False) -> list[Path]:
    from ppy_compiler.ir import read

    from ppy_b200 import artifacts

    written = []
    for name in names:
        source = GOLDEN / f"{name}.ppyir"
        if not source.exists():
            continue
        module = read(source)
        written += artifacts.write_module(module, HERE / name, compile_library=compile_library)
    return written


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference", type=Path, required=True)
    parser.add_argument("names", nargs="*", default=list(MODULES))
    options = parser.parse_args()
    sys.path.insert(0, str(options.reference / "src"))
    sys.path.insert(0, str(REPO))
    for path in regenerate(options.names):
        print(path.relative_to(REPO))


if __name__ == "__main__":
    main()
