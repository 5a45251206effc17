"""Two devices driven from two threads of one process: the runtime binds a device per calling
thread (ppyb200_init), and every kernel's launch set-up -- the shared-memory attribute, the
resident cluster count -- is kept per device, so each device's first GEMM, attention and
layernorm launch correctly whichever device went first. Needs 2 GPUs (skipped on one)."""

from __future__ import annotations

import threading

import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
F = pytest.importorskip("torch.nn.functional")


def _work(device: int, results: dict, errors: list, start: threading.Barrier) -> None:
    try:
        from ppy_b200 import gpt2, runtime

        torch.cuda.set_device(device)
        assert runtime.library().ppyb200_init(device) == 0
        stream = torch.cuda.Stream(device=device)
        runtime.set_stream(stream)
        lib = runtime.library()
        gpt2._bind(lib)
        g = torch.Generator(device=f"cuda:{device}").manual_seed(device)
        with torch.cuda.stream(stream):
            a = torch.randn(512, 768, device=f"cuda:{device}", generator=g).to(torch.bfloat16)
            w = torch.randn(2304, 768, device=f"cuda:{device}", generator=g).to(torch.bfloat16)
            c = torch.empty(512, 2304, device=f"cuda:{device}")
            qkv = (0.5 * torch.randn(2 * 256, 3 * 768, device=f"cuda:{device}",
                                     generator=g)).to(torch.bfloat16)
            out = torch.empty(2 * 256, 768, device=f"cuda:{device}", dtype=torch.bfloat16)
        stream.synchronize()
        start.wait()  # both threads launch their first kernels at the same time
        assert lib.ppyb200_matmul_bf16_kmajor(a.data_ptr(), w.data_ptr(), None, c.data_ptr(),
                                              512, 2304, 768) == 0, runtime.last_error()
        assert lib.ppyb200_attention_causal_bf16(qkv.data_ptr(), out.data_ptr(), 2, 256, 12,
                                                 64) == 0, runtime.last_error()
        model = gpt2.GPT2(gpt2.Config(layers=1), seed=device, device=f"cuda:{device}")
        ids = torch.randint(0, 50257, (1, 128), device=f"cuda:{device}", generator=g)
        with torch.cuda.stream(stream):
            logits = model.forward(ids)
        stream.synchronize()
        assert model.status() == 0
        ref_mm = a.float() @ w.float().t()
        q, k, v = qkv.float().split(768, dim=1)
        shape = lambda t: t.reshape(2, 256, 12, 64).transpose(1, 2)  # noqa: E731
        ref_att = F.scaled_dot_product_attention(shape(q), shape(k), shape(v), is_causal=True)
        ref_att = ref_att.transpose(1, 2).reshape(512, 768)
        results[device] = (float((c - ref_mm).abs().max() / ref_mm.abs().max()),
                           float((out.float() - ref_att).abs().max() / ref_att.abs().max()),
                           bool(torch.isfinite(logits).all()), torch.cuda.current_device())
    except BaseException as exc:  # noqa: BLE001 - reported by the test
        errors.append((device, repr(exc)))
        start.abort()


def test_two_devices_from_two_threads():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    results: dict = {}
    errors: list = []
    start = threading.Barrier(2)
    threads = [threading.Thread(target=_work, args=(d, results, errors, start)) for d in (0, 1)]
    for t in threads:
        t.start()
    for t in threads:
        t.join(timeout=300)
    assert not errors, errors
    for device in (0, 1):
        mm, att, finite, bound = results[device]
        assert mm <= 1e-5 and att <= 2e-2 and finite and bound == device, results[device]
