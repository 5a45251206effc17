"""PPy source over `ppy.Tensor` reaches the backend: the `b200_tensor` plugin
(ppy_b200.tensor_plugin) types the calls of `ppy_b200.tensor` into tensor-dialect operations,
as the fixture plugin of the reference's tests/test_common_tensor_lowering.py:69-149 types its
own, and the backend's first pass turns the tensor parameters into buffers. The real `ppy`
CLI in a subprocess, with the plugin and the backend installed as entry points, as
tests/test_backend_api.py does; CPU only (nvcc cross-compiles)."""

from __future__ import annotations

import importlib.machinery
import importlib.util
import json
import os
import subprocess
import sys
import textwrap
from pathlib import Path

import numpy as np
import pytest

from conftest import GOLDEN, REFERENCE, REPO

pytestmark = pytest.mark.reference


def _site(tmp_path: Path) -> Path:
    site = tmp_path / "site"
    info = site / "ppy_b200-0.1.0.dist-info"
    info.mkdir(parents=True)
    (info / "METADATA").write_text("Metadata-Version: 2.1\nName: ppy-b200\nVersion: 0.1.0\n")
    (info / "entry_points.txt").write_text(
        "[ppy.backends]\nb200 = ppy_b200:create_backend\n\n"
        "[ppy.backend-formats]\nb200-cu = b200\nb200-plan = b200\n\n"
        "[ppy.plugins]\nb200_tensor = ppy_b200.tensor_plugin:create_plugin\n")
    return site


def _project(tmp_path: Path, name: str, source: str, plugin: bool = True) -> Path:
    root = tmp_path / "proj"
    root.mkdir()
    text = f'[project]\nname = "{name}"\nversion = "0"\n'
    if plugin:
        text += "\n[tool.ppy.plugins.b200_tensor]\n"
    (root / "pyproject.toml").write_text(text)
    (root / f"{name}.ppy").write_text(source)
    return root


def _ppy(cwd: Path, site: Path, *args: str) -> subprocess.CompletedProcess:
    env = dict(os.environ)
    env["PYTHONPATH"] = os.pathsep.join([str(site), str(REPO), str(REFERENCE / "src")])
    return subprocess.run([sys.executable, "-m", "ppy_compiler", *args], cwd=cwd,
                          capture_output=True, text=True, env=env, check=False, timeout=600)


def test_ppy_source_gelu_builds_one_map_kernel(ppy_compiler, tmp_path):
    root = _project(tmp_path, "gelu_source", (GOLDEN / "gelu_source.ppy").read_text())
    done = _ppy(root, _site(tmp_path), "build", "gelu_source.ppy", "--backend", "b200", "-o",
                "out")
    assert done.returncode == 0, done.stdout + done.stderr
    manifest = json.loads((root / "out" / "gelu_source.json").read_text())
    (fn,) = manifest["functions"]
    assert fn["kernels"] == ["map"]  # every operation of the chain in one kernel
    assert [(p["name"], p["role"]) for p in fn["params"]] == [
        ("a", "in"), ("b", "in"), ("c", "in"), ("out", "out")]
    assert (root / "out" / "gelu_source.so").exists()


def test_without_the_plugin_the_calls_have_no_types(ppy_compiler, tmp_path):
    root = _project(tmp_path, "gelu_source", (GOLDEN / "gelu_source.ppy").read_text(),
                    plugin=False)
    done = _ppy(root, _site(tmp_path), "build", "gelu_source.ppy", "--backend", "b200", "-o",
                "out")
    assert done.returncode != 0


def test_rows_and_matmul_from_source(ppy_compiler, tmp_path):
    source = textwrap.dedent("""
        import ppy
        import ppy_b200.tensor as bt


        def softmax_rows(x: ppy.Tensor[ppy.f32, (512, 256)],
                         out: ppy.Mut[ppy.Tensor[ppy.f32, (512, 256)]]) -> None:
            m = bt.max(x, axes=(1,), keepdims=True)
            e = bt.exp(bt.sub(x, m))
            s = bt.sum(e, axes=(1,), keepdims=True)
            bt.assign(out, bt.div(e, s))


        def linear_relu(a: ppy.Tensor[ppy.bf16, (256, 128)], w: ppy.Tensor[ppy.bf16, (128, 64)],
                        bias: ppy.Tensor[ppy.f32, (64,)],
                        out: ppy.Mut[ppy.Tensor[ppy.f32, (256, 64)]]) -> None:
            # bf16 operands, f32 products: converts the matmul kernel reads itself
            y = bt.add(bt.matmul(bt.convert(a, dtype="f32"), bt.convert(w, dtype="f32")), bias)
            bt.assign(out, bt.maximum(y, bt.full(0.0)))
    """)
    root = _project(tmp_path, "layers", source)
    done = _ppy(root, _site(tmp_path), "build", "layers.ppy", "--backend", "b200", "-o", "out")
    assert done.returncode == 0, done.stdout + done.stderr
    manifest = json.loads((root / "out" / "layers.json").read_text())
    kernels = {fn["name"]: fn["kernels"] for fn in manifest["functions"]}
    assert kernels["layers_softmax_rows"] == ["row"]
    assert kernels["layers_linear_relu"][0] == "matmul"


def test_cpython_runs_the_same_source_as_numpy(ppy_compiler):
    """The Python meaning of the source (ppy_b200/tensor.py) against the oracle's GELU."""
    import oracle

    sys.path.insert(0, str(REFERENCE / "src"))
    loader = importlib.machinery.SourceFileLoader("gelu_source", str(GOLDEN / "gelu_source.ppy"))
    spec = importlib.util.spec_from_loader("gelu_source", loader)
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)
    rng = np.random.default_rng(0)
    n = 1 << 20
    a, b, c = (rng.uniform(-4, 4, n).astype(np.float32) for _ in range(3))
    out = np.empty(n, np.float32)
    module.gelu_chain(a, b, c, out)
    ref = oracle.gelu_chain(a, b, c)
    scale = np.maximum(np.abs(ref), 1.0)
    assert float(np.max(np.abs(out - ref) / scale)) <= 1e-5
