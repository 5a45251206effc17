"""Regenerate the prebuilt modules from the fixtures in tests/golden/.

Each `tests/golden/<name>.ppyir` is canonical IR as PPy's shared passes hand it to a
backend; this runs the b200 backend's translation on it -- the same code
`ppy build <name>.ppyir --backend b200` runs -- and writes `<name>/<name>.cu` and
`<name>/<name>.json` here. Each `tests/golden/<name>.ppy` is PPy source over `ppy.Tensor`
values: it goes through PPy's frontend with the `b200_tensor` plugin, the shared passes and the
backend's own passes first, as `ppy build <name>.ppy --backend b200` takes it. The libraries (`<name>.so`) are compiled from those by
`__graft_entry__.build()` or on first load. Needs PPy's compiler importable
(`--reference /path/to/PPy`).
"""

from __future__ import annotations

import argparse
import os
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
GOLDEN = REPO / "tests" / "golden"
MODULES = ("gelu", "rows", "chain", "reductions", "collatz", "matmul", "matmul_bf16",
           "matmul_bf16_8192", "matmul_f32_4096", "gpt2_layernorm", "gelu_source", "views",
           "collatz_threads", "parallel_math")


def regenerate(names=MODULES, compile_library: bool = False) -> list[Path]:
    from ppy_compiler.ir import read

    from ppy_b200 import artifacts

    written = []
    for name in names:
        source = GOLDEN / f"{name}.ppyir"
        if source.exists():
            module = read(source)
        elif (GOLDEN / f"{name}.ppy").exists():
            module = from_source(GOLDEN / f"{name}.ppy")
        else:
            continue
        written += artifacts.write_module(module, HERE / name, compile_library=compile_library)
    return written


def from_source(path: Path):
    """The canonical IR of PPy source `path` as the b200 backend receives it (after its passes)."""
    from ppy_compiler.driver.ir_pipeline import canonical_ir_modules
    from ppy_compiler.driver.pipeline import analyze_paths, open_project

    from ppy_b200.backend import B200Backend
    from ppy_b200.tensor_plugin import TensorPlugin

    import tempfile

    # a project of its own, so that `ppy_b200.tensor` is the plugin's module and not a source
    # file of this repository's project
    with tempfile.TemporaryDirectory() as scratch:
        root = Path(scratch)
        (root / "pyproject.toml").write_text(
            f'[project]\nname = "{path.stem}"\nversion = "0"\n\n[tool.ppy.plugins.b200_tensor]\n')
        copy = root / path.name
        copy.write_text(path.read_text())
        project = open_project(copy)
        project.plugins.register(TensorPlugin())
        bundle = analyze_paths(project, [copy], backend="b200")
        if bundle.diagnostics.has_errors():
            raise SystemExit("\n".join(str(d) for d in bundle.diagnostics.sorted()))
        (module,) = canonical_ir_modules(bundle, backend=B200Backend()).values()
    return module


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference", type=Path, default=os.environ.get("PPY_REFERENCE"),
                        required="PPY_REFERENCE" not in os.environ,
                        help="a PPy checkout (default: $PPY_REFERENCE)")
    parser.add_argument("names", nargs="*", default=list(MODULES))
    options = parser.parse_args()
    sys.path.insert(0, str(options.reference / "src"))
    sys.path.insert(0, str(REPO))
    for path in regenerate(options.names):
        print(path.relative_to(REPO))


if __name__ == "__main__":
    main()
