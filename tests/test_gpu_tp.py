"""The tensor-parallel GPT-2 forward (ppy_b200.gpt2_tp) on 2, 4 and 8 GPUs, one process each --
one group of 2, two data-parallel groups of 2, one group of 4, two groups of 4, and a group of
one on a single GPU (the whole vocabulary in one rank's pitched logits rows) -- with the
row-parallel exchange over NCCL or fused into the GEMM over NVLink: every rank's logits slice
of its group's sequences against the torch float32 forward of the same weights (the
reference's ATen block, examples/46_gpt2/gpt2.ppy:18-57) and against the one-GPU forward of
the b200 kernels. Each case is skipped on a box with fewer GPUs. On one GPU: the exchange's
kernels with two emulated ranks, and its bounded wait giving up."""

from __future__ import annotations

import os
import socket
import sys

import pytest

from conftest import REPO

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank: int, world: int, port: int, queue, tp: int = 0, exchange: str = "nccl") -> None:
    import datetime

    import torch.distributed as dist

    sys.path.insert(0, str(REPO))
    from oracle import gpt2 as oracle_gpt2
    from ppy_b200 import gpt2, gpt2_tp, runtime

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120))
    try:
        runtime.init(rank)
        runtime.set_stream(torch.cuda.current_stream())
        cfg = gpt2.Config(layers=2)
        dp, tp_size = gpt2_tp.hybrid_layout(world, cfg, tp)
        group, dpi = gpt2_tp.hybrid_groups(tp_size)
        tp = gpt2_tp.GPT2TensorParallel(cfg, seed=0, group=group, exchange=exchange)
        g = torch.Generator(device="cuda").manual_seed(5)
        ids = torch.randint(0, 50257, (2 * dp, 256), device="cuda", generator=g)
        ids = ids[2 * dpi:2 * dpi + 2].contiguous()  # this group's sequences
        got = tp.forward(ids)
        again = tp.forward(ids)  # a second forward: the exchange's epochs and parities move on
        torch.cuda.synchronize()
        status = tp.status()
        same = bool(torch.equal(got, again))
        tp.close()
        full = gpt2.GPT2(cfg, seed=0)
        v0, v1 = tp.shard.vocab
        one_gpu = full.forward(ids)[..., v0:v1]
        ref = oracle_gpt2.forward(full, ids)[..., v0:v1]
        torch.cuda.synchronize()
        diff = (got - ref).double()
        queue.put((rank, status, float(diff.abs().max() / ref.abs().max()),
                   float(diff.norm() / ref.double().norm()),
                   float((got - one_gpu).abs().max() / one_gpu.abs().max()), same))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,tp,exchange", [(1, 0, "nccl"), (2, 0, "nccl"), (2, 0, "nvlink"),
                                               (4, 2, "nccl"), (4, 2, "nvlink"),
                                               (4, 0, "nvlink"), (8, 0, "nccl")])
def test_tensor_parallel_forward(world, tp, exchange):
    if not torch.cuda.is_available():
        pytest.fail("a GPU test ran without a CUDA device")
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = torch.multiprocessing.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, queue, tp, exchange))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        assert p.exitcode == 0
    for _ in range(world):
        rank, status, worst, norm, vs_one, same = queue.get(timeout=10)
        assert same, rank  # the same ids give the same logits on the second forward
        assert status == 0, rank
        # logits, tensor-relative (2e-2, the bf16 GEMM paths' tolerance)
        assert worst <= 2e-2 and norm <= 2e-2, (rank, worst, norm)
        # against one GPU: the same kernels, partial products summed in another order
        assert vs_one <= 1e-2, (rank, vs_one)


# ---------------------------------------------------------------- the exchange's kernels on one GPU


def _exchange_lib():
    from ppy_b200 import gpt2_tp, runtime

    if not torch.cuda.is_available():
        pytest.fail("a GPU test ran without a CUDA device")
    runtime.init(0)
    runtime.set_stream(torch.cuda.current_stream())
    lib = runtime.library()
    gpt2_tp._bind_exchange(lib)
    return lib


def test_exchange_kernels_with_two_ranks_on_one_gpu():
    """Two ranks' steps, one after the other on one stream, with every slot on this GPU: each
    partial product lands in its slot of both buffers, the signals raise both flag arrays,
    and each accumulate gives x + bias + p0 + p1 (in that order: the two results agree bit
    for bit)."""
    import ctypes

    lib = _exchange_lib()
    m, n, k = 300, 768, 128
    g = torch.Generator(device="cuda").manual_seed(3)
    a = [torch.randn(m, k, device="cuda", generator=g).to(torch.bfloat16) for _ in range(2)]
    w = [torch.randn(n, k, device="cuda", generator=g).to(torch.bfloat16) for _ in range(2)]
    bias = torch.randn(n, device="cuda", generator=g)
    x0 = torch.randn(m, n, device="cuda", generator=g)
    buffers = [torch.zeros(2, m, n, device="cuda") for _ in range(2)]  # [slot, M, N] per rank
    flags = [torch.zeros(8, dtype=torch.int32, device="cuda") for _ in range(2)]
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    flag_set = (ctypes.c_void_p * 2)(*[f.data_ptr() for f in flags])
    for r in range(2):
        slots = (ctypes.c_void_p * 2)(*[b[r].data_ptr() for b in buffers])
        assert lib.ppyb200_tp_partial_scatter(a[r].data_ptr(), w[r].data_ptr(), slots, 2, m, n,
                                              k, status.data_ptr()) == 0
        assert lib.ppyb200_tp_signal(flag_set, 2, r, 1) == 0
    xs = [x0.clone(), x0.clone()]
    for r in range(2):
        assert lib.ppyb200_tp_accumulate(xs[r].data_ptr(), bias.data_ptr(),
                                         buffers[r].data_ptr(), flags[r].data_ptr(), 2, m, n, 1,
                                         status.data_ptr()) == 0
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    assert flags[0][:2].tolist() == [1, 1] and flags[1][:2].tolist() == [1, 1]
    parts = [(a[r].float() @ w[r].float().t()) for r in range(2)]
    for r in range(2):
        assert torch.allclose(buffers[0][r], parts[r], rtol=1e-4, atol=1e-3)
        assert torch.equal(buffers[0][r], buffers[1][r])
    want = x0 + (bias + parts[0] + parts[1])
    assert torch.allclose(xs[0], want, rtol=1e-4, atol=1e-3)
    assert torch.equal(xs[0], xs[1])


def test_reduce_scatter_exchange_with_three_ranks_on_one_gpu():
    """The reduce-scatter form, three ranks' steps one after the other on one stream (every
    buffer on this GPU), over 301 rows (blocks of 101, 101, 99): each rank's x ends equal, bit
    for bit, to the all-slot form's x + bias + p0 + p1 + p2."""
    import ctypes

    lib = _exchange_lib()
    ranks, m, n, k = 3, 301, 768, 128
    rows = (m + ranks - 1) // ranks
    g = torch.Generator(device="cuda").manual_seed(5)
    a = [torch.randn(m, k, device="cuda", generator=g).to(torch.bfloat16) for _ in range(ranks)]
    w = [torch.randn(n, k, device="cuda", generator=g).to(torch.bfloat16) for _ in range(ranks)]
    bias = torch.randn(n, device="cuda", generator=g)
    x0 = torch.randn(m, n, device="cuda", generator=g)
    exchange = [torch.zeros(ranks, rows, n, device="cuda") for _ in range(ranks)]
    gather = [torch.zeros(ranks, rows, n, device="cuda") for _ in range(ranks)]
    flags = [torch.zeros(16, dtype=torch.int32, device="cuda") for _ in range(ranks)]
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    first = (ctypes.c_void_p * ranks)(*[f.data_ptr() for f in flags])
    second = (ctypes.c_void_p * ranks)(*[f.data_ptr() + 32 for f in flags])
    for r in range(ranks):
        slots = (ctypes.c_void_p * ranks)(*[e[r].data_ptr() for e in exchange])
        assert lib.ppyb200_tp_partial_reduce_scatter(a[r].data_ptr(), w[r].data_ptr(), slots,
                                                     ranks, m, n, k, status.data_ptr()) == 0
        assert lib.ppyb200_tp_signal(first, ranks, r, 1) == 0
    xs = [x0.clone() for _ in range(ranks)]
    for r in range(ranks):
        peers = (ctypes.c_void_p * ranks)(*[gt[r].data_ptr() for gt in gather])
        assert lib.ppyb200_tp_reduce_block(xs[r].data_ptr(), bias.data_ptr(),
                                           exchange[r].data_ptr(), peers, flags[r].data_ptr(),
                                           ranks, r, m, n, 1, status.data_ptr()) == 0
        assert lib.ppyb200_tp_signal(second, ranks, r, 1) == 0
    for r in range(ranks):
        assert lib.ppyb200_tp_gather_blocks(xs[r].data_ptr(), gather[r].data_ptr(),
                                            flags[r].data_ptr() + 32, ranks, r, m, n, 1,
                                            status.data_ptr()) == 0
    # the all-slot form on the same operands
    full = torch.zeros(ranks, m, n, device="cuda")
    one = torch.zeros(16, dtype=torch.int32, device="cuda")
    for r in range(ranks):
        slots = (ctypes.c_void_p * ranks)(*([full[r].data_ptr()] * ranks))
        assert lib.ppyb200_tp_partial_scatter(a[r].data_ptr(), w[r].data_ptr(), slots, 1, m, n,
                                              k, status.data_ptr()) == 0
    one[:ranks] = 1
    want = x0.clone()
    assert lib.ppyb200_tp_accumulate(want.data_ptr(), bias.data_ptr(), full.data_ptr(),
                                     one.data_ptr(), ranks, m, n, 1, status.data_ptr()) == 0
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    parts = [(a[r].float() @ w[r].float().t()) for r in range(ranks)]
    assert torch.allclose(want, x0 + (bias + parts[0] + parts[1] + parts[2]), rtol=1e-4,
                          atol=1e-3)
    for r in range(ranks):
        assert torch.equal(xs[r], want), r


def test_exchange_wait_gives_up_and_raises_the_status():
    """A flag that nothing raises: the accumulate's bounded wait (about 2 s) gives up, raises
    the status word to 2 and leaves x alone; the context stays usable."""
    lib = _exchange_lib()
    m, n = 64, 768
    x = torch.randn(m, n, device="cuda")
    before = x.clone()
    exchange = torch.ones(2, m, n, device="cuda")
    flags = torch.zeros(8, dtype=torch.int32, device="cuda")
    flags[0] = 5  # one rank has signalled, the other never does
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    assert lib.ppyb200_tp_accumulate(x.data_ptr(), None, exchange.data_ptr(), flags.data_ptr(),
                                     2, m, n, 5, status.data_ptr()) == 0
    torch.cuda.synchronize()
    assert int(status.item()) == 2
    assert torch.equal(x, before)
    assert float((x + 1).sum()) == float((before + 1).sum())  # the device still runs work
