"""The drop-in boundary: PPy finds, loads and builds with the b200 backend through its own
Backend API, as tests/test_backend_api.py:191-249 of the reference installs a backend -- a
distribution with a `ppy.backends` entry point on PYTHONPATH, and the real CLI in a
subprocess. CPU only: nvcc cross-compiles for sm_100a without a GPU."""

from __future__ import annotations

import json
import os
import subprocess
import sys
import textwrap
from pathlib import Path

import pytest

from conftest import GOLDEN, PREBUILT, REFERENCE, REPO

pytestmark = pytest.mark.reference


def _site(tmp_path: Path) -> Path:
    site = tmp_path / "site"
    info = site / "ppy_b200-0.1.0.dist-info"
    info.mkdir(parents=True)
    (info / "METADATA").write_text("Metadata-Version: 2.1\nName: ppy-b200\nVersion: 0.1.0\n")
    (info / "entry_points.txt").write_text(
        "[ppy.backends]\nb200 = ppy_b200:create_backend\n\n"
        "[ppy.backend-formats]\nb200-cu = b200\nb200-plan = b200\n")
    return site


def _ppy(cwd: Path, site: Path, *args: str) -> subprocess.CompletedProcess:
    env = dict(os.environ)
    env["PYTHONPATH"] = os.pathsep.join([str(site), str(REPO), str(REFERENCE / "src")])
    return subprocess.run([sys.executable, "-m", "ppy_compiler", *args], cwd=cwd,
                          capture_output=True, text=True, env=env, check=False, timeout=600)


@pytest.fixture
def project(tmp_path, ppy_compiler):
    root = tmp_path / "proj"
    root.mkdir()
    (root / "pyproject.toml").write_text('[project]\nname = "proj"\nversion = "0"\n')
    return root, _site(tmp_path)


def test_ppy_builds_a_ppyir_module_with_the_b200_backend(project):
    root, site = project
    (root / "gelu.ppyir").write_text((GOLDEN / "gelu.ppyir").read_text())
    done = _ppy(root, site, "build", "gelu.ppyir", "--backend", "b200", "-o", "out")
    assert done.returncode == 0, done.stdout + done.stderr
    out = root / "out"
    assert (out / "gelu.cu").exists() and (out / "gelu.so").exists()
    manifest = json.loads((out / "gelu.json").read_text())
    assert manifest["format"] == "ppy-b200/1" and manifest["arch"] == "sm_100a"
    (fn,) = manifest["functions"]
    assert fn["name"] == "gelu_chain" and fn["kernels"] == ["map"]
    assert [p["role"] for p in fn["params"]] == ["in", "in", "in", "out"]


COLLATZ = """
from ppy import parallel


def collatz_sum(lo: int, hi: int) -> int:
    total = 0
    for start in parallel.range(lo, hi):
        x = start
        steps = 0
        while x != 1:
            if x % 2 == 0:
                x = x // 2
            else:
                x = 3 * x + 1
            steps += 1
        total += steps
    return total
"""


def _parallel_project(root: Path) -> None:
    (root / "pyproject.toml").write_text('[project]\nname = "proj"\nversion = "0"\n\n'
                                         '[tool.ppy.parallel]\nbackend = "openmp"\n')
    (root / "collatz.ppy").write_text(COLLATZ)


def test_emit_gives_the_generated_cuda_of_a_ppy_source(project):
    root, site = project
    _parallel_project(root)
    done = _ppy(root, site, "emit", "b200-cu", "collatz.ppy")
    assert done.returncode == 0, done.stdout + done.stderr
    assert "dev_collatz_collatz_sum__par1" in done.stdout
    assert "PPYB200_LOOP_LIMIT" in done.stdout


def test_ppy_builds_a_ppy_source_with_a_parallel_range(project):
    root, site = project
    _parallel_project(root)
    done = _ppy(root, site, "build", "collatz.ppy", "--backend", "b200", "-o", "out")
    assert done.returncode == 0, done.stdout + done.stderr
    manifest = json.loads((root / "out" / "collatz.json").read_text())
    (fn,) = manifest["functions"]
    assert fn["symbol"] == "ppy_collatz_collatz_sum" and fn["kind"] == "scalar"
    assert (root / "out" / "collatz.so").exists()


def test_doctor_lists_the_backend(project):
    root, site = project
    done = _ppy(root, site, "doctor")
    assert "b200" in done.stdout + done.stderr


def test_unsupported_ir_is_refused_with_the_reason(project):
    root, site = project
    # rows of a symbolic length: the backend names what it cannot take
    (root / "t.ppyir").write_text(textwrap.dedent('''\
        ppyir 1
        module @t
        dialect core 1
        dialect tensor 1

        func @rowsum(%a: buffer<f32>, %out: buffer<f32>) -> i64 {
        ^entry:
            %0 = tensor.load %a : tensor.tensor<f32, 4, N>
            %1 = tensor.reduce %0 {axes = [1], keepdims = false, op = "add"} : tensor.tensor<f32, 4>
            tensor.store %1, %out
            %2 = core.const 0 : i64
            core.ret %2
        }
        '''))
    done = _ppy(root, site, "build", "t.ppyir", "--backend", "b200", "-o", "out")
    assert done.returncode != 0
    text = done.stdout + done.stderr
    assert "E1802" in text and "b200" in text and "reduction" in text and "symbolic" in text


def test_committed_prebuilt_modules_are_what_the_backend_generates(ppy_compiler, tmp_path):
    """ppy_b200/prebuilt/ is regenerated output; the backend still produces it byte for byte."""
    from ppy_compiler.ir import read

    from ppy_b200 import artifacts
    from ppy_b200.prebuilt.regenerate import from_source

    for directory in sorted(p for p in PREBUILT.iterdir() if p.is_dir()):
        name = directory.name
        if (GOLDEN / f"{name}.ppyir").exists():
            module = read(GOLDEN / f"{name}.ppyir")
        else:  # PPy source over ppy.Tensor, through the b200_tensor plugin
            module = from_source(GOLDEN / f"{name}.ppy")
        written = artifacts.write_module(module, tmp_path / name, compile_library=False)
        for path in written:
            assert path.read_text() == (directory / path.name).read_text(), path.name


COLLATZ_SOURCE = textwrap.dedent("""
    import ppy


    def collatz_steps(n: int) -> int:
        steps = 0
        while n != 1:
            if n % 2 == 0:
                n = n // 2
            else:
                n = 3 * n + 1
            steps += 1
        return steps


    def collatz_sum(lo: int, hi: int) -> int:
        total = 0
        for i in ppy.parallel.range(lo, hi):
            total += collatz_steps(i)
        return total
""")


def test_parallel_range_source_builds_on_both_routes(project):
    """PPy source with ppy.parallel.range (examples/35_parallel_range). Under the default
    threads route the range arrives split into host-thread chunks (`concurrency.spawn`); the
    backend's pass gives the loop its range back (ppy_b200.passes.thread_chunks_to_ranges) and
    builds the same reduce kernel as under the openmp setting, which keeps the range whole."""
    root, site = project
    (root / "collatz.ppy").write_text(COLLATZ_SOURCE)
    kernels = []
    for route in ("threads", "openmp"):
        if route == "openmp":
            with (root / "pyproject.toml").open("a") as f:
                f.write('\n[tool.ppy.parallel]\nbackend = "openmp"\n')
        done = _ppy(root, site, "build", "collatz.ppy", "--backend", "b200", "-o", route)
        assert done.returncode == 0, done.stdout + done.stderr
        manifest = json.loads((root / route / "collatz.json").read_text())
        kernels.append({fn["name"]: fn["kernels"] for fn in manifest["functions"]})
    assert kernels[0] == kernels[1]
    assert kernels[0]["collatz_collatz_sum"] == ["reduce"]


def test_thread_chunks_become_the_range_again(ppy_compiler):
    """The threads route's IR of the Collatz program (tests/golden/collatz_threads.ppyir):
    after the pass no concurrency op is left, and each loop is the parallel op the openmp
    route's IR (tests/golden/collatz.ppyir) has, with the same callee and reduction."""
    from ppy_compiler.ir import read, verify

    from ppy_b200.passes import thread_chunks_to_ranges

    module = read(GOLDEN / "collatz_threads.ppyir")
    assert thread_chunks_to_ranges(module)
    assert not verify(module)
    ops = [op for fn in module.functions.values() if not fn.is_declaration
           for op in fn.operations()]
    assert not [op for op in ops if op.dialect == "concurrency"]
    got = sorted((op.name, op.attributes["callee"].name, str(op.attributes.get("op")))
                 for op in ops if op.dialect == "parallel")
    assert got == [("parallel.for", "collatz_collatz_steps__par2", "None"),
                   ("parallel.reduce", "collatz_collatz_sum__par1", "add")]
    assert not thread_chunks_to_ranges(module)  # nothing left to do
