"""Loading and calling what a b200 build wrote.

`load(path)` reads a module's manifest (`<module>.json`) and binds its library; every
IR function becomes a callable with the reference's native calling convention
(backend/llvm/from_ir.py:1-13, as tests/test_tensor_fusion.py:269-282 calls it): buffers
as (pointer, length), scalars by value, the result through a slot, an int32 status back.

    module = load("build/gelu.json")
    status, value = module.gelu_chain(a, b, c, out)            # NumPy arrays in host memory
    status, value = module.device.gelu_chain(ta, tb, tc, tout)  # torch CUDA tensors

A status of STATUS_FALLBACK means a guard failed and the caller reruns the function
in CPython, as for the LLVM backend; STATUS_RAISED raises `B200Error` with the CUDA
error. There is no CPU path here: without the libraries or a GPU the calls fail.
"""

from __future__ import annotations

import ctypes
import json
import threading
from dataclasses import dataclass
from pathlib import Path

from . import toolchain

__all__ = ["B200Error", "STATUS_FALLBACK", "STATUS_OK", "STATUS_RAISED", "Module", "library",
           "load", "set_stream"]

STATUS_OK = 0
STATUS_FALLBACK = 1
STATUS_RAISED = -1

_CTYPES = {
    "f32": ctypes.c_float, "f64": ctypes.c_double, "bf16": ctypes.c_uint16,
    "i64": ctypes.c_int64, "index": ctypes.c_int64, "i32": ctypes.c_int32,
    "i16": ctypes.c_int16, "i8": ctypes.c_int8, "u64": ctypes.c_uint64,
    "u32": ctypes.c_uint32, "u16": ctypes.c_uint16, "u8": ctypes.c_uint8, "bool": ctypes.c_bool,
}
_NUMPY = {"f32": "float32", "f64": "float64", "bf16": "uint16", "i64": "int64", "index": "int64",
          "i32": "int32", "i16": "int16", "i8": "int8", "u64": "uint64", "u32": "uint32",
          "u16": "uint16", "u8": "uint8", "bool": "bool"}


class B200Error(RuntimeError):
    """The device or the runtime failed; the message says how."""


_lock = threading.Lock()
_library: ctypes.CDLL | None = None


def library() -> ctypes.CDLL:
    """libppyb200.so, loaded once with its symbols global (the modules resolve them)."""
    global _library
    with _lock:
        if _library is not None:
            return _library
        path = toolchain.RUNTIME_LIBRARY
        if not path.exists():
            raise B200Error(f"{path} is not built: run `python -c 'import __graft_entry__ as g; "
                            "g.build()'` or ppy_b200.toolchain.build_runtime()")
        lib = ctypes.CDLL(str(path), mode=ctypes.RTLD_GLOBAL)
        lib.ppyb200_last_error.restype = ctypes.c_char_p
        lib.ppyb200_init.argtypes = [ctypes.c_int32]
        lib.ppyb200_set_stream.argtypes = [ctypes.c_void_p]
        lib.ppyb200_stream.restype = ctypes.c_void_p
        lib.ppyb200_launches.restype = ctypes.c_uint64
        lib.ppyb200_device_allocations.restype = ctypes.c_uint64
        lib.ppyb200_count_launches.argtypes = [ctypes.c_uint64]
        lib.ppyb200_copy_rows_to_host.argtypes = [ctypes.c_void_p, ctypes.c_int64,
                                                  ctypes.c_void_p, ctypes.c_int64,
                                                  ctypes.c_int64, ctypes.c_int64]
        lib.ppyb200_scratch.restype = ctypes.c_void_p
        lib.ppyb200_scratch.argtypes = [ctypes.c_int64]
        lib.ppyb200_device_buffer.restype = ctypes.c_void_p
        lib.ppyb200_device_buffer.argtypes = [ctypes.c_int64]
        lib.ppyb200_release_buffer.argtypes = [ctypes.c_void_p]
        _library = lib
        return lib


def last_error() -> str:
    return library().ppyb200_last_error().decode(errors="replace")


def init(device: int = 0) -> None:
    if library().ppyb200_init(int(device)) != STATUS_OK:
        raise B200Error(f"device {device}: {last_error()}")


#: cudaStreamLegacy: the default stream, spelled so that it is not mistaken for "none".
_LEGACY_STREAM = 0x1


def set_stream(stream) -> None:
    """Launch this thread's calls on `stream`: a torch.cuda.Stream or a raw cudaStream_t
    handle (torch's default stream, handle 0, is the legacy default stream), or None for
    the runtime's own non-blocking stream of the device."""
    if stream is None:
        library().ppyb200_set_stream(ctypes.c_void_p(0))
        return
    handle = int(getattr(stream, "cuda_stream", stream) or 0)
    library().ppyb200_set_stream(ctypes.c_void_p(handle or _LEGACY_STREAM))


def device_allocations() -> int:
    """cudaMalloc calls the runtime library has made since it loaded."""
    return int(library().ppyb200_device_allocations())


def count_launches(count: int) -> None:
    """Add `count` kernels to the launch counter (launches a CUDA graph replays)."""
    library().ppyb200_count_launches(ctypes.c_uint64(count))


def copy_rows_to_host(host, device) -> None:
    """Copy the rows of a 2-D (or batched) CUDA tensor `device` into the pinned host tensor
    `host` of the same shape and dtype, both with unit stride along the last axis and evenly
    spaced rows, with one strided copy on the current stream (asynchronous)."""
    rows = device.numel() // device.shape[-1]
    row_bytes = device.shape[-1] * device.element_size()
    if tuple(host.shape) != tuple(device.shape) or host.dtype != device.dtype:
        raise B200Error("copy_rows_to_host: the same shape and dtype on both sides")
    pitches = []
    for t in (host, device):
        if t.stride(-1) != 1 or (t.dim() > 2 and t.stride(-3) != t.shape[-2] * t.stride(-2)):
            raise B200Error("copy_rows_to_host: unit stride along rows, rows evenly spaced")
        pitches.append(t.stride(-2) * t.element_size())
    status = library().ppyb200_copy_rows_to_host(
        ctypes.c_void_p(host.data_ptr()), ctypes.c_int64(pitches[0]),
        ctypes.c_void_p(device.data_ptr()), ctypes.c_int64(pitches[1]),
        ctypes.c_int64(row_bytes), ctypes.c_int64(rows))
    if status != STATUS_OK:
        raise B200Error(last_error())


def launches() -> int:
    """Kernels launched through the runtime and its modules since the library loaded."""
    return int(library().ppyb200_launches())


@dataclass(frozen=True)
class Result:
    status: int
    value: int

    def __iter__(self):
        return iter((self.status, self.value))


def _host_buffer(value, dtype: str):
    """(address, length) of a host array: a NumPy array or a CPU torch tensor."""
    if hasattr(value, "data_ptr") and hasattr(value, "is_cuda"):
        if value.is_cuda:
            raise B200Error("a host call takes host memory; use module.device.<fn> for CUDA tensors")
        if not value.is_contiguous():
            raise B200Error("buffers are contiguous")
        return value.data_ptr(), value.numel()
    import numpy as np

    array = value
    if not isinstance(array, np.ndarray):
        raise B200Error(f"a buffer is a NumPy array or a torch tensor, not {type(value).__name__}")
    if not array.flags.c_contiguous:
        raise B200Error("buffers are C-contiguous")
    if array.dtype != np.dtype(_NUMPY[dtype]):
        raise B200Error(f"a buffer<{dtype}> takes {_NUMPY[dtype]} elements, not {array.dtype}")
    return array.ctypes.data, array.size


def _device_buffer(value):
    if isinstance(value, tuple) and len(value) == 2:
        return int(value[0]), int(value[1])
    if hasattr(value, "data_ptr"):
        if not value.is_cuda:
            raise B200Error("a device call takes CUDA tensors")
        if not value.is_contiguous():
            raise B200Error("buffers are contiguous")
        return value.data_ptr(), value.numel()
    raise B200Error("a device buffer is a CUDA tensor or an (address, length) pair")


class Function:
    """One exported IR function, host or device flavour."""

    def __init__(self, lib: ctypes.CDLL, entry: dict, device: bool) -> None:
        self.entry = entry
        self.device = device
        self.name = entry["name"]
        symbol = entry["symbol"] + ("__device" if device else "")
        self._fn = getattr(lib, symbol)
        argtypes = []
        for p in entry["params"]:
            element = _CTYPES[p["dtype"]]
            if p["kind"] == "buffer":
                argtypes += [ctypes.c_void_p, ctypes.c_int64]
            elif p["kind"] == "ptr":
                argtypes.append(ctypes.c_void_p)
            else:
                argtypes.append(element)
        argtypes.append(ctypes.POINTER(ctypes.c_int64))
        self._fn.argtypes = argtypes
        self._fn.restype = ctypes.c_int32

    def atoms(self, args) -> list:
        params = self.entry["params"]
        if len(args) != len(params):
            raise TypeError(f"{self.name} takes {len(params)} arguments, not {len(args)}")
        atoms = []
        for p, value in zip(params, args):
            if p["kind"] == "buffer":
                pointer, length = _device_buffer(value) if self.device else _host_buffer(
                    value, p["dtype"])
                atoms += [ctypes.c_void_p(pointer), length]
            elif p["kind"] == "ptr":
                pointer = value.data_ptr() if hasattr(value, "data_ptr") else int(value)
                atoms.append(ctypes.c_void_p(pointer))
            else:
                atoms.append(value)
        return atoms

    def __call__(self, *args) -> Result:
        slot = ctypes.c_int64(0)
        status = int(self._fn(*self.atoms(args), ctypes.byref(slot)))
        if status == STATUS_RAISED:
            raise B200Error(f"{self.name}: {last_error()}")
        return Result(status, int(slot.value))


class _Namespace:
    pass


class Module:
    """A built module: `module.<fn>` (host memory) and `module.device.<fn>`."""

    def __init__(self, manifest_path: Path) -> None:
        self.path = manifest_path
        self.manifest = json.loads(manifest_path.read_text(encoding="utf-8"))
        if self.manifest.get("format") != "ppy-b200/1":
            raise B200Error(f"{manifest_path} is not a b200 manifest")
        library()
        so = manifest_path.parent / self.manifest["library"]
        source = manifest_path.parent / self.manifest["source"]
        if source.exists():
            toolchain.build_module(source, so)  # rebuilt only when stale
        if not so.exists():
            raise B200Error(f"{so} is missing and its source is not beside it")
        # RTLD_LOCAL: a module's symbols stay its own (two builds may export one name)
        self.lib = ctypes.CDLL(str(so), mode=ctypes.RTLD_LOCAL)
        self.device = _Namespace()
        self.functions: dict[str, Function] = {}
        for entry in self.manifest["functions"]:
            host = Function(self.lib, entry, device=False)
            self.functions[entry["name"]] = host
            setattr(self, entry["name"], host)
            setattr(self.device, entry["name"], Function(self.lib, entry, device=True))


def load(path) -> Module:
    """A built module from its manifest (`<dir>/<module>.json`)."""
    path = Path(path)
    if path.is_dir():
        manifests = sorted(path.glob("*.json"))
        if len(manifests) != 1:
            raise B200Error(f"{path} holds {len(manifests)} manifests; name one")
        path = manifests[0]
    return Module(path)
