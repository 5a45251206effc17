"""The C ABI: every function include/*.h declares is exported by the built libraries,
and the libraries load on a machine without a GPU (no compute is called here)."""

from __future__ import annotations

import ctypes
import json
import re

import pytest

from conftest import PREBUILT, REPO

DECL = re.compile(r"^[A-Za-z_][\w\s\*]*?\b(ppyb200_\w+)\s*\(", re.M)


def declared() -> list[str]:
    names = []
    for header in sorted((REPO / "include").glob("*.h")):
        text = re.sub(r"/\*.*?\*/", "", header.read_text(), flags=re.S)
        names += DECL.findall(text)
    return sorted(set(names))


def test_header_declares_the_runtime():
    names = declared()
    assert "ppyb200_init" in names and "ppyb200_last_error" in names and len(names) >= 15


def test_runtime_library_exports_every_declared_symbol():
    from ppy_b200 import runtime, toolchain

    toolchain.build_runtime()
    lib = runtime.library()
    missing = [name for name in declared() if not hasattr(lib, name)]
    assert not missing, missing
    assert lib.ppyb200_abi_version() == 1


def test_runtime_reports_no_device_without_one():
    from ppy_b200 import runtime

    torch = pytest.importorskip("torch")
    if torch.cuda.is_available():
        pytest.skip("a device is present")
    assert runtime.library().ppyb200_device_count() == 0


@pytest.mark.parametrize("name", sorted(p.name for p in PREBUILT.iterdir() if p.is_dir()))
def test_prebuilt_module_exports_its_manifest(name):
    from ppy_b200 import runtime, toolchain

    # a directory holds one module, its files named after the IR module (collatz_threads/
    # holds collatz.*: the same program as collatz/, from PPy's threads route)
    (path,) = (PREBUILT / name).glob("*.json")
    manifest = json.loads(path.read_text())
    so = toolchain.build_module(path.with_suffix(".cu"), path.with_suffix(".so"))
    runtime.library()
    lib = ctypes.CDLL(str(so), mode=ctypes.RTLD_GLOBAL)
    for fn in manifest["functions"]:
        assert hasattr(lib, fn["symbol"]) and hasattr(lib, fn["symbol"] + "__device")
