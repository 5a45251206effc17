"""nvcc for sm_100a: building the runtime library and each module's library.

Everything is compiled ahead of time into shared libraries in the source tree (the
runtime) or the build output directory (modules); nothing is compiled at run time
unless a module's library is missing beside its source.
"""

from __future__ import annotations

import hashlib
import os
import shutil
import subprocess
from pathlib import Path

PACKAGE = Path(__file__).resolve().parent
CSRC = PACKAGE / "csrc"
INCLUDE = PACKAGE.parent / "include"
RUNTIME_SOURCES = ("ppyb200_runtime.cu", "gemm_sm100.cu", "gpt2.cu", "noalloc.cu",
                   "tp_exchange.cu", "probes.cu")
RUNTIME_LIBRARY = PACKAGE / "libppyb200.so"
ARCH = "sm_100a"
GENCODE = ["-gencode", "arch=compute_100a,code=sm_100a"]


class ToolchainError(RuntimeError):
    """nvcc is missing or refused a source; the message carries its output."""


def nvcc() -> str | None:
    found = shutil.which("nvcc")
    if found:
        return found
    default = Path("/usr/local/cuda/bin/nvcc")
    return str(default) if default.exists() else None


def nvcc_version() -> str:
    tool = nvcc()
    if tool is None:
        return ""
    out = subprocess.run([tool, "--version"], capture_output=True, text=True, check=False).stdout
    for line in out.splitlines():
        if "release" in line:
            return line.strip()
    return out.strip().splitlines()[-1] if out.strip() else ""


def flags() -> list[str]:
    return [*GENCODE, "-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
            "-diag-suppress", "177,550",
            "-Xcompiler", "-fPIC", "-shared", f"-I{CSRC}", f"-I{INCLUDE}"]


def compile_shared(sources: list[Path], output: Path, extra: list[str] | None = None) -> Path:
    tool = nvcc()
    if tool is None:
        raise ToolchainError("nvcc is not on PATH or in /usr/local/cuda/bin")
    output.parent.mkdir(parents=True, exist_ok=True)
    tmp = output.with_suffix(output.suffix + f".{os.getpid()}.tmp")
    command = [tool, *flags(), *(extra or []), "-o", str(tmp), *map(str, sources)]
    done = subprocess.run(command, capture_output=True, text=True, check=False)
    if done.returncode != 0:
        raise ToolchainError(f"nvcc failed ({' '.join(command)}):\n{done.stdout}\n{done.stderr}")
    os.replace(tmp, output)
    return output


def _digest(paths: list[Path]) -> str:
    h = hashlib.sha256()
    for p in paths:
        h.update(p.read_bytes())
    h.update(" ".join(flags()).encode())
    return h.hexdigest()[:16]


def build_runtime(force: bool = False) -> Path:
    """libppyb200.so from csrc/, rebuilt when a source or header changed."""
    sources = [CSRC / s for s in RUNTIME_SOURCES if (CSRC / s).exists()]
    headers = sorted(CSRC.glob("*.cuh")) + [INCLUDE / "ppyb200.h"]
    stamp = RUNTIME_LIBRARY.with_suffix(".so.stamp")
    digest = _digest(sources + headers)
    if not force and RUNTIME_LIBRARY.exists() and stamp.exists() and stamp.read_text() == digest:
        return RUNTIME_LIBRARY
    compile_shared(sources, RUNTIME_LIBRARY)
    stamp.write_text(digest)
    return RUNTIME_LIBRARY


def build_module(source: Path, output: Path, force: bool = False) -> Path:
    """A module's generated source into its library, linked against the runtime."""
    headers = sorted(CSRC.glob("*.cuh")) + [INCLUDE / "ppyb200.h"]
    stamp = output.with_suffix(".so.stamp")
    digest = _digest([source] + headers)
    if not force and output.exists() and stamp.exists() and stamp.read_text() == digest:
        return output
    runtime = build_runtime()
    compile_shared([source], output,
                   ["-Xcompiler", "-fvisibility=hidden", f"-L{runtime.parent}", "-lppyb200",
                    f"-Xlinker=-rpath,{runtime.parent}", "-Xlinker=-Bsymbolic"])
    stamp.write_text(digest)
    return output
