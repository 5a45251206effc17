"""The matmul entry points through the C ABI, against a float64 evaluation of the same
bf16 inputs (NumPy has no bf16; torch rounds them). Tolerance for the bf16 paths: 2e-2
relative on outputs, written here as |C - ref| <= 2e-2 * max(|ref|, rms(ref)); the
tensor-core kernel accumulates in f32 and lands far inside it."""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

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
    for name in ("ppyb200_matmul_bf16", "ppyb200_matmul_bf16_kmajor"):
        getattr(lib, name).argtypes = [ctypes.c_void_p] * 4 + [ctypes.c_int64] * 3
        getattr(lib, name).restype = ctypes.c_int32
    lib.ppyb200_matmul_bf16_kmajor_ld.argtypes = [ctypes.c_void_p] * 4 + [ctypes.c_int64] * 4
    lib.ppyb200_matmul_bf16_kmajor_ld.restype = ctypes.c_int32
    lib.ppyb200_transpose_bf16.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64,
                                           ctypes.c_int64]
    lib.ppyb200_set_gemm_form.argtypes = [ctypes.c_int32]
    lib.ppyb200_set_gemm_form.restype = ctypes.c_int32
    return lib


def _operands(m, n, k, seed=0, bias=True):
    g = torch.Generator().manual_seed(seed)
    a = (torch.randn(m, k, generator=g) / k ** 0.5).to(torch.bfloat16)
    b = (torch.randn(k, n, generator=g) / k ** 0.5).to(torch.bfloat16)
    c = (0.02 * torch.randn(n, generator=g)) if bias else None
    return a, b, c


def _reference(a, b, bias):
    ref = a.double() @ b.double()
    if bias is not None:
        ref = ref + bias.double()
    return ref.numpy()


def _check(out, ref, rel=2e-2):
    out = out.cpu().double().numpy()
    scale = np.maximum(np.abs(ref), np.sqrt(np.mean(ref ** 2)))
    err = np.abs(out - ref) / scale
    assert float(err.max()) <= rel, float(err.max())
    return float(err.max())


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr() if t is not None else 0)


@pytest.mark.parametrize("m,n,k", [(128, 256, 64), (256, 512, 192), (1024, 1024, 1024),
                                   (384, 768, 768)])
def test_tensor_core_matmul_matches_float64(lib, m, n, k):
    a, b, bias = _operands(m, n, k)
    da, db, dbias = a.cuda(), b.cuda(), bias.cuda()
    out = torch.full((m, n), float("nan"), device="cuda")
    status = lib.ppyb200_matmul_bf16(_ptr(da), _ptr(db), _ptr(dbias), _ptr(out), m, n, k)
    torch.cuda.synchronize()
    assert status == 0
    err = _check(out, _reference(a, b, bias))
    assert err < 1e-4  # f32 accumulation of bf16 products: far inside the bound


def test_kmajor_entry_and_no_bias(lib):
    m, n, k = 256, 256, 128
    a, b, _ = _operands(m, n, k, seed=1, bias=False)
    da, bt = a.cuda(), b.t().contiguous().cuda()  # held: a pointer alone keeps nothing alive
    out = torch.empty((m, n), device="cuda")
    assert lib.ppyb200_matmul_bf16_kmajor(_ptr(da), _ptr(bt), None, _ptr(out), m, n, k) == 0
    torch.cuda.synchronize()
    _check(out, _reference(a, b, None), rel=1e-4)


def test_kmajor_refuses_k_not_a_multiple_of_64(lib):
    a = torch.zeros(128, 96, dtype=torch.bfloat16, device="cuda")
    bt = torch.zeros(256, 96, dtype=torch.bfloat16, device="cuda")
    out = torch.zeros(128, 256, device="cuda")
    assert lib.ppyb200_matmul_bf16_kmajor(_ptr(a), _ptr(bt), None, _ptr(out), 128, 256, 96) == 1


@pytest.mark.parametrize("m,n,k", [(100, 70, 64), (1, 50257, 128), (300, 520, 192),
                                   (200, 50257, 64), (130, 131, 128)])
def test_tensor_cores_take_ragged_m_and_n(lib, m, n, k):
    """Edge tiles: TMA zero-fills past M and N, the epilogue stores only inside."""
    a, b, bias = _operands(m, n, k, seed=6)
    da, dbt, dbias = a.cuda(), b.t().contiguous().cuda(), bias.cuda()
    out = torch.full((m + 1, n), 7.0, device="cuda")  # one row past C must stay untouched
    assert lib.ppyb200_matmul_bf16_kmajor(_ptr(da), _ptr(dbt), _ptr(dbias), _ptr(out), m, n,
                                          k) == 0
    torch.cuda.synchronize()
    _check(out[:m], _reference(a, b, bias), rel=1e-4)
    assert torch.all(out[m] == 7.0)


@pytest.mark.parametrize("m,n,k", [(256, 256, 64), (512, 768, 768), (300, 520, 192),
                                   (1, 50257, 128), (130, 131, 128), (1000, 2304, 3072)])
def test_cta_pairs_match_single_ctas(lib, m, n, k):
    """The 2-CTA kernel (256 x 256 tiles, tcgen05.mma.cta_group::2) against the one-CTA kernel
    and float64: aligned, ragged and deep-K shapes, bias added, one row past C untouched."""
    a, b, bias = _operands(m, n, k, seed=9)
    da, dbt, dbias = a.cuda(), b.t().contiguous().cuda(), bias.cuda()
    outs = []
    try:
        for form in (2, 1):  # one CTA per tile, then CTA pairs
            assert lib.ppyb200_set_gemm_form(form) in (0, 1, 2)
            out = torch.full((m + 1, n), 7.0, device="cuda")
            assert lib.ppyb200_matmul_bf16_kmajor(_ptr(da), _ptr(dbt), _ptr(dbias), _ptr(out),
                                                  m, n, k) == 0
            torch.cuda.synchronize()
            outs.append(out)
    finally:
        lib.ppyb200_set_gemm_form(0)
    one, pair = outs
    assert torch.all(pair[m] == 7.0)
    _check(pair[:m], _reference(a, b, bias), rel=1e-4)
    assert torch.allclose(pair, one, rtol=1e-5, atol=1e-5)


def test_gemm_form_refuses_other_values(lib):
    assert lib.ppyb200_set_gemm_form(3) == -1
    assert lib.ppyb200_set_gemm_form(0) == 0  # by shape, the default


@pytest.mark.parametrize("offset", [4, 36, 1])
def test_logit_rows_at_any_offset(lib, offset):
    """C inside a larger buffer, rows of 50257 floats starting 16-byte aligned (offsets 4 and
    36 floats, not on a 128-byte line) or only 4-byte aligned (offset 1): every element of C
    lands once and nothing either side of it is touched."""
    m, n, k = 260, 50257, 128
    a, b, bias = _operands(m, n, k, seed=7)
    da, dbt, dbias = a.cuda(), b.t().contiguous().cuda(), bias.cuda()
    buf = torch.full((offset + m * n + 64,), 7.0, device="cuda")
    out = buf[offset:offset + m * n].view(m, n)
    assert lib.ppyb200_matmul_bf16_kmajor(_ptr(da), _ptr(dbt), _ptr(dbias), _ptr(out), m, n,
                                          k) == 0
    torch.cuda.synchronize()
    _check(out, _reference(a, b, bias), rel=1e-4)
    assert torch.all(buf[:offset] == 7.0) and torch.all(buf[offset + m * n:] == 7.0)


@pytest.mark.parametrize("m,n,k,ldc", [(260, 50257, 128, 50272), (260, 25129, 768, 25152),
                                        (300, 520, 192, 544),
                                        (256, 256, 64, 257), (130, 131, 128, 131)])
def test_rows_at_a_pitch(lib, m, n, k, ldc):
    """C in rows ldc floats apart: the values of the contiguous call, bit for bit, and the
    columns N .. ldc-1 of every row untouched (128-byte lines -- the LM head's 50257 and a
    two-rank vocabulary slice's 25129 -- odd pitches, ldc == N)."""
    a, b, bias = _operands(m, n, k, seed=10)
    da, dbt, dbias = a.cuda(), b.t().contiguous().cuda(), bias.cuda()
    rows = torch.full((m + 1, ldc), 7.0, device="cuda")
    dense = torch.empty((m, n), device="cuda")
    assert lib.ppyb200_matmul_bf16_kmajor_ld(_ptr(da), _ptr(dbt), _ptr(dbias), _ptr(rows), ldc,
                                             m, n, k) == 0
    assert lib.ppyb200_matmul_bf16_kmajor(_ptr(da), _ptr(dbt), _ptr(dbias), _ptr(dense), m, n,
                                          k) == 0
    torch.cuda.synchronize()
    assert torch.equal(rows[:m, :n], dense)
    assert torch.all(rows[:m, n:] == 7.0) and torch.all(rows[m] == 7.0)
    _check(dense, _reference(a, b, bias), rel=1e-4)


def test_pitch_below_n_is_refused(lib):
    a = torch.zeros(128, 64, dtype=torch.bfloat16, device="cuda")
    bt = torch.zeros(256, 64, dtype=torch.bfloat16, device="cuda")
    out = torch.zeros(128, 256, device="cuda")
    assert lib.ppyb200_matmul_bf16_kmajor_ld(_ptr(a), _ptr(bt), None, _ptr(out), 255, 128, 256,
                                             64) == -1


@pytest.mark.parametrize("m,n,k", [(100, 70, 33), (1, 256, 64), (129, 257, 65)])
def test_ragged_shapes_run_on_cuda_cores(lib, m, n, k):
    a, b, bias = _operands(m, n, k, seed=2)
    da, db, dbias = a.cuda(), b.cuda(), bias.cuda()
    out = torch.empty((m, n), device="cuda")
    status = lib.ppyb200_matmul_bf16(_ptr(da), _ptr(db), _ptr(dbias), _ptr(out), m, n, k)
    torch.cuda.synchronize()
    assert status == 0
    _check(out, _reference(a, b, bias), rel=1e-4)


def test_transpose(lib):
    b = torch.randn(300, 70).to(torch.bfloat16).cuda()
    bt = torch.empty(70, 300, dtype=torch.bfloat16, device="cuda")
    assert lib.ppyb200_transpose_bf16(_ptr(b), _ptr(bt), 300, 70) == 0
    torch.cuda.synchronize()
    assert torch.equal(bt, b.t())


def test_bench_size_matmul_properties(lib):
    """8192^3 (the benchmark shape): the whole output against an f32 matmul of the same
    bf16-rounded operands (cuBLAS, TF32 off), spot rows against float64, and linearity in B."""
    m = n = k = 8192
    a, b, bias = _operands(m, n, k, seed=3)
    da, db, dbias = a.cuda(), b.cuda(), bias.cuda()
    out = torch.empty((m, n), device="cuda")
    assert lib.ppyb200_matmul_bf16(_ptr(da), _ptr(db), _ptr(dbias), _ptr(out), m, n, k) == 0
    torch.cuda.synchronize()
    tf32 = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        whole = torch.addmm(dbias, da.float(), db.float())
    finally:
        torch.backends.cuda.matmul.allow_tf32 = tf32
    scale = torch.maximum(whole.abs(), whole.pow(2).mean().sqrt())
    worst = float(((out - whole).abs() / scale).max())
    assert worst <= 1e-4, worst  # two f32 accumulations of the same products, other orders
    del whole, scale
    rows = torch.tensor([0, 1, 127, 128, 4095, 8191])
    ref = (a[rows].double() @ b.double() + bias.double()).numpy()
    _check(out[rows.cuda()], ref, rel=1e-4)
    # linearity: A @ (2B) is exactly 2 (A @ B) (scaling by 2 is exact in bf16 and f32)
    plain = torch.empty_like(out)
    twice = torch.empty_like(out)
    db2 = db * 2
    assert lib.ppyb200_matmul_bf16(_ptr(da), _ptr(db), None, _ptr(plain), m, n, k) == 0
    assert lib.ppyb200_matmul_bf16(_ptr(da), _ptr(db2), None, _ptr(twice), m, n, k) == 0
    torch.cuda.synchronize()
    assert torch.equal(twice, 2 * plain)


# ---------------------------------------------------------------- through built modules


def _module(name):
    from conftest import PREBUILT
    from ppy_b200 import runtime

    return runtime.load(PREBUILT / name / f"{name}.json")


def test_f32_matmul_module_matches_the_reference(lib):
    """matmul.ppyir (f32, 64x96 @ 96x80 + bias) against PPy's LLVM JIT output."""
    from conftest import GOLDEN, within

    d = np.load(GOLDEN / "matmul.npz")
    module = _module("matmul")
    out = np.zeros_like(d["out"])
    status, _ = module.matmul_bias(d["a"].ravel(), d["b"].ravel(), d["bias"], out.ravel())
    assert status == int(d["status"]) == 0
    within(out, d["out"])


@pytest.mark.parametrize("m", [256, 100, 0])
def test_bf16_matmul_module(lib, m):
    """matmul_bf16.ppyir: whole tiles on tensor cores, other row counts on CUDA cores."""
    module = _module("matmul_bf16")
    a, b, bias = _operands(max(m, 1), 256, 128, seed=4)
    a = a[:m]
    out = np.zeros((m, 256), np.float32)
    status, _ = module.matmul_bias_bf16(a.view(torch.int16).numpy().view(np.uint16).ravel(),
                                        b.view(torch.int16).numpy().view(np.uint16).ravel(),
                                        bias.numpy(), out.ravel())
    assert status == 0
    if m:
        _check(torch.from_numpy(out), _reference(a, b, bias), rel=1e-4)


def test_bench_shape_module_rows(lib):
    module = _module("matmul_bf16_8192")
    a, b, bias = _operands(128, 8192, 8192, seed=5)
    da, db, dbias = a.cuda(), b.cuda(), bias.cuda()
    out = torch.empty((128, 8192), device="cuda")
    assert module.device.matmul_bias_bf16(da, db, dbias, out).status == 0
    torch.cuda.synchronize()
    _check(out, _reference(a, b, bias), rel=1e-4)


# ---------------------------------------------------------------- f32 operands (three tf32 products)
#
# ppyb200_matmul_f32 computes A_hi B_hi + A_hi B_lo + A_lo B_hi on the tensor cores (x_hi = x
# rounded to tf32, x_lo = the rest rounded to tf32). Tolerance: the north star's 1e-5 relative
# for fp32 reductions, per element against max(|ref|, rms(ref)) of a float64 evaluation.


def _f32_operands(m, n, k, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    a = torch.randn(m, k, device="cuda", generator=g) / max(k, 1) ** 0.5
    b = torch.randn(k, n, device="cuda", generator=g) / max(k, 1) ** 0.5
    bias = 0.02 * torch.randn(n, device="cuda", generator=g)
    return a, b, bias


def _matmul_f32(lib, a, b, bias, m, n, k):
    lib.ppyb200_matmul_f32.argtypes = [ctypes.c_void_p] * 4 + [ctypes.c_int64] * 3
    lib.ppyb200_matmul_f32.restype = ctypes.c_int32
    c = torch.full((m, n), float("nan"), device="cuda")
    assert lib.ppyb200_matmul_f32(_ptr(a), _ptr(b), _ptr(bias), _ptr(c), m, n, k) == 0
    torch.cuda.synchronize()
    return c


def _f32_reference(a, b, bias):
    ref = a.double() @ b.double()
    return ref + bias.double() if bias is not None else ref


def _check_f32(c, ref, rel=1e-5):
    scale = torch.maximum(ref.abs(), ref.pow(2).mean().sqrt())
    err = float(((c.double() - ref).abs() / scale).max())
    assert err <= rel, err
    return err


def test_f32_matmul_4096_cube_against_float64(lib):
    """The fp32-input variant at its benchmark size, whole output against float64."""
    m = n = k = 4096
    a, b, bias = _f32_operands(m, n, k, seed=1)
    c = _matmul_f32(lib, a, b, bias, m, n, k)
    _check_f32(c, _f32_reference(a, b, bias))


@pytest.mark.parametrize("m,n,k", [(1, 1, 1), (100, 200, 50), (300, 513, 77), (257, 255, 1000),
                                   (64, 96, 80), (1024, 1024, 4096)])
def test_f32_matmul_ragged_shapes(lib, m, n, k):
    a, b, bias = _f32_operands(m, n, k, seed=2)
    c = _matmul_f32(lib, a, b, bias, m, n, k)
    _check_f32(c, _f32_reference(a, b, bias))


def test_f32_matmul_empty_k_gives_the_bias(lib):
    _, _, bias = _f32_operands(64, 96, 1, seed=3)
    a = torch.empty(64, 0, device="cuda")
    b = torch.empty(0, 96, device="cuda")
    c = _matmul_f32(lib, a, b, bias, 64, 96, 0)
    assert torch.equal(c, bias.expand(64, 96))


@pytest.mark.parametrize("form", [1, 2])
def test_f32_matmul_pairs_and_single_ctas_agree(lib, form):
    m, n, k = 512, 768, 1024
    a, b, bias = _f32_operands(m, n, k, seed=4)
    before = lib.ppyb200_set_gemm_form(form)
    try:
        c = _matmul_f32(lib, a, b, bias, m, n, k)
    finally:
        lib.ppyb200_set_gemm_form(before)
    _check_f32(c, _f32_reference(a, b, bias))


def test_f32_matmul_non_finite_inputs_follow_ieee(lib):
    """An infinity or a NaN among the inputs: C is recomputed with f32 FMAs, so infinities
    stay infinities (a tf32 split would give NaN where inf meets a zero low part)."""
    m, n, k = 96, 130, 70
    a, b, bias = _f32_operands(m, n, k, seed=5)
    b = b.abs() + 0.25  # positive columns: inf * b keeps its sign
    a[3, 10] = float("inf")
    a[7, 0] = float("-inf")
    a[11, 5] = float("nan")
    c = _matmul_f32(lib, a, b, bias, m, n, k)
    ref = _f32_reference(a, b, bias)
    assert torch.equal(torch.isnan(c), torch.isnan(ref))
    assert torch.equal(torch.isinf(c), torch.isinf(ref))
    inf = torch.isinf(ref)
    assert torch.equal(torch.sign(c[inf]), torch.sign(ref[inf]).float())
    finite = torch.isfinite(ref)
    scale = ref[finite].pow(2).mean().sqrt()
    assert float(((c[finite].double() - ref[finite]).abs() / torch.maximum(
        ref[finite].abs(), scale)).max()) <= 1e-5


@pytest.mark.parametrize("m,n,k", [(4096, 768, 768), (32768, 768, 1536), (300, 1152, 128),
                                   (100, 768, 64), (4096, 768, 3072)])
def test_192_wide_tiles_match_256_wide_bit_for_bit(lib, m, n, k):
    """N a multiple of 192: the default form takes 192-wide tiles where they need fewer
    waves at shallow K (pick_tile_n; K = 3072 keeps 256); every output element still sums
    its K products in the same order,
    so the result equals the 256-wide tiles' (forms pinned by ppyb200_set_gemm_form) exactly,
    for the column and the four-column-quads epilogues."""
    a, b, bias = _operands(m, n, k, seed=11)
    da, dbt, dbias = a.cuda(), b.t().contiguous().cuda(), bias.cuda()
    ref = None
    for ldc in (n, n + 4):  # quads (rows on 16-byte boundaries) at K < 2048, columns beyond
        outs = {}
        for form in (0, 1, 2):
            out = torch.full((m, ldc), 5.0, device="cuda")
            before = lib.ppyb200_set_gemm_form(form)
            try:
                assert lib.ppyb200_matmul_bf16_kmajor_ld(_ptr(da), _ptr(dbt), _ptr(dbias),
                                                         _ptr(out), ldc, m, n, k) == 0
            finally:
                lib.ppyb200_set_gemm_form(before)
            torch.cuda.synchronize()
            outs[form] = out
        pinned = outs[1] if m >= 256 else outs[2]
        assert torch.equal(outs[0], pinned)
        assert torch.all(outs[0][:, n:] == 5.0)
        if ref is None:
            ref = _reference(a[:512], b, bias)
        _check(outs[0][:512, :n], ref, rel=1e-4)
