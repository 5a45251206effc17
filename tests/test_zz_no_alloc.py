"""The entry point that allocates nothing, against the allocating one.

`ppyb200_colmax_abs_f32_noalloc` serves callers that cannot allocate device memory when
they call (their memory is reserved once at start-up, or belongs to another framework's
allocator): its partial results live in a fixed device array instead of the scratch arena
the generated `colmax` grows on demand. Both compute max over rows of |x| per column; a max
is exact, so the results must agree bit for bit -- on two calls in a row, the second on
a different shape, since the array keeps the first call's contents. This file sorts last
so that a run stopping at the first failure has already run every other test.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

from conftest import PREBUILT

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def lib():
    from ppy_b200 import runtime

    if not torch.cuda.is_available():
        pytest.fail("a GPU test ran without a CUDA device")
    runtime.init(0)
    runtime.set_stream(torch.cuda.current_stream())
    lib = runtime.library()
    lib.ppyb200_colmax_abs_f32_noalloc.argtypes = [ctypes.c_void_p, ctypes.c_int64,
                                                   ctypes.c_int64, ctypes.c_void_p]
    lib.ppyb200_colmax_abs_f32_noalloc.restype = ctypes.c_int32
    return lib


def _allocating(x):
    from ppy_b200 import runtime

    module = runtime.load(PREBUILT / "reductions" / "reductions.json")
    out = torch.empty(64, device="cuda")
    assert module.device.colmax(x.view(-1), out).status == 0
    return out


def test_no_alloc_colmax_matches_the_allocating_entry_point_twice(lib):
    g = torch.Generator(device="cuda").manual_seed(7)
    shapes = [(100_000, 64), (777, 64)]
    for rows, cols in shapes:
        x = torch.randn(rows, cols, device="cuda", generator=g)
        x[rows // 2, 5] = float("nan")  # a NaN wins its column in both
        expected = _allocating(x)
        out = torch.full((cols,), 3.0, device="cuda")
        status = lib.ppyb200_colmax_abs_f32_noalloc(x.data_ptr(), rows, cols, out.data_ptr())
        torch.cuda.synchronize()
        assert status == 0
        assert torch.equal(torch.nan_to_num(out, nan=-1.0), torch.nan_to_num(expected, nan=-1.0))
        assert torch.isnan(out[5]) and torch.isnan(expected[5])


def test_no_alloc_colmax_allocates_nothing_once_the_device_is_bound(lib):
    """The property the entry point exists for. ppyb200_init (in the fixture) loads its code
    and static array onto the device; from then on calls on shapes it has not seen allocate
    nothing: neither this library's cudaMalloc count nor the device's free memory moves."""
    from ppy_b200 import runtime

    g = torch.Generator(device="cuda").manual_seed(11)
    shapes = [(123_457, 17), (3, 262_144), (4096, 1000)]
    inputs = [torch.randn(rows, cols, device="cuda", generator=g) for rows, cols in shapes]
    outs = [torch.empty(cols, device="cuda") for _, cols in shapes]
    warm = torch.randn(512, 64, device="cuda", generator=g)
    warm_out = torch.empty(64, device="cuda")
    assert lib.ppyb200_colmax_abs_f32_noalloc(warm.data_ptr(), 512, 64, warm_out.data_ptr()) == 0
    torch.cuda.synchronize()
    before = (runtime.device_allocations(), torch.cuda.mem_get_info()[0])
    for x, out, (rows, cols) in zip(inputs, outs, shapes):
        assert lib.ppyb200_colmax_abs_f32_noalloc(x.data_ptr(), rows, cols, out.data_ptr()) == 0
    torch.cuda.synchronize()
    after = (runtime.device_allocations(), torch.cuda.mem_get_info()[0])
    assert after == before
    for x, out in zip(inputs, outs):
        assert torch.equal(out, x.abs().amax(dim=0))


def test_no_alloc_colmax_refuses_rows_wider_than_its_array(lib):
    from ppy_b200 import runtime

    x = torch.zeros(1, device="cuda")
    out = torch.zeros(1, device="cuda")
    status = lib.ppyb200_colmax_abs_f32_noalloc(x.data_ptr(), 1, 262145, out.data_ptr())
    assert status == -1
    assert "262144" in runtime.last_error()
