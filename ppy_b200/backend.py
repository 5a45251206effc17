"""The `b200` backend: PPy's Backend API v1 (backend/base.py:219-295) for B200 GPUs.

Installed as the entry point `b200 = "ppy_b200:create_backend"` of the
`ppy.backends` group (backend/registry.py:42), it is reached by
`ppy build X --backend b200` and `ppy build X.ppyir --backend b200`
(driver/commands.py:609-736). It receives canonical IR after the shared passes, refuses
what it cannot map in `validate`, and `build` writes, per module, generated CUDA C++,
its sm_100a library and a manifest (see `artifacts`). Running the result is the
runtime's business (`ppy_b200.runtime.load`), as the Backend API leaves it
(docs/internals/backends.md, "Limitations").
"""

from __future__ import annotations

import hashlib
import json
from collections.abc import Mapping
from pathlib import Path

from ppy_compiler.backend import (
    Backend,
    BackendContext,
    BackendPassRegistrar,
    BackendValidationError,
    BuildResult,
    EmitFormat,
    ToolchainStatus,
)
from ppy_compiler.ir.passes import Pass, PassContext

from . import __version__, artifacts
from .passes import CommonTensorsToBuffers, ReductionsToTrailingAxes, ThreadChunksToRanges
from .scalar_c import Unsupported
from .toolchain import ARCH, CSRC, nvcc, nvcc_version

__all__ = ["B200Backend", "KernelPlanRemarks"]


def _sources_digest() -> str:
    h = hashlib.sha256()
    package = Path(__file__).resolve().parent
    for path in sorted(package.glob("*.py")) + sorted(CSRC.glob("*")):
        if path.is_file():
            h.update(path.name.encode())
            h.update(path.read_bytes())
    return h.hexdigest()[:16]


class KernelPlanRemarks(Pass):
    """Backend-stage pass: says, per function, which kernels the build will make.

    It changes nothing; its remarks (`ppy build --report-opt`) show how the tensor
    operations FuseTensor left are regrouped -- e.g. the four reductions and four
    elementwise groups of a softmax followed by a layernorm become one row kernel.
    """

    name = "b200-kernel-plan"

    def run(self, module, ctx: PassContext) -> bool:
        try:
            planned, _source = artifacts.plan_and_source(module)
        except (Unsupported, ValueError):
            return False
        for note in planned.notes:
            ctx.remark(f"b200: {note}")
        return False


class B200Backend(Backend):
    name = "b200"
    api_version = 1

    def fingerprint(self) -> str:
        return hashlib.sha256(
            json.dumps([type(self).__qualname__, self.api_version, __version__, ARCH,
                        nvcc_version(), _sources_digest()]).encode()
        ).hexdigest()

    def emit_formats(self) -> tuple[EmitFormat, ...]:
        return (
            EmitFormat("b200-cu", ".cu", description="CUDA C++ for sm_100a (B200)",
                       requires_toolchain=False),
            EmitFormat("b200-plan", ".json", description="the b200 kernel manifest",
                       requires_toolchain=False),
        )

    def register_passes(self, passes: BackendPassRegistrar) -> None:
        passes.add(CommonTensorsToBuffers)
        passes.add(ReductionsToTrailingAxes)
        passes.add(ThreadChunksToRanges)
        passes.add(KernelPlanRemarks)

    def validate(self, module, context: BackendContext) -> None:
        try:
            artifacts.plan_and_source(module)
        except Unsupported as error:
            raise BackendValidationError(self.name, error.what,
                                         capability=error.capability) from error
        except ValueError as error:
            raise BackendValidationError(self.name, str(error)) from error

    def emit(self, module, format: str, context: BackendContext) -> str:  # noqa: A002
        planned, source = artifacts.plan_and_source(module)
        if format == "b200-cu":
            return source
        if format == "b200-plan":
            return json.dumps(artifacts.manifest(planned), indent=1) + "\n"
        return super().emit(module, format, context)

    def build(self, modules: Mapping[str, object], output: Path,
              context: BackendContext) -> BuildResult:
        written: list[Path] = []
        notes: list[str] = []
        for name, module in modules.items():
            try:
                paths = artifacts.write_module(module, output)
            except Unsupported as error:
                raise BackendValidationError(self.name, error.what,
                                             capability=error.capability) from error
            written.extend(paths)
            notes.append(f"{name}: built for {ARCH}")
        return BuildResult(tuple(written), tuple(notes))

    def toolchain_status(self) -> ToolchainStatus:
        tool = nvcc()
        if tool is None:
            return ToolchainStatus(False, "missing nvcc (CUDA 12.8+ for sm_100a)")
        return ToolchainStatus(True, f"{nvcc_version()}, {ARCH}")
