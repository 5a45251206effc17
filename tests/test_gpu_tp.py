"""The tensor-parallel GPT-2 forward (ppy_b200.gpt2_tp) on 2, 4 and 8 GPUs, one process each over
NCCL -- one group of 2, two data-parallel groups of 2, two groups of 4: every rank's logits
slice of its group's sequences against the torch float32 forward of the same weights (the
reference's ATen block, examples/46_gpt2/gpt2.ppy:18-57) and against the one-GPU forward of
the b200 kernels. Each case is skipped on a box with fewer GPUs."""

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


def _rank(rank: int, world: int, port: int, queue, tp: int = 0) -> None:
    import datetime

    import torch.distributed as dist

    sys.path.insert(0, str(REPO))
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
        tp = gpt2_tp.GPT2TensorParallel(cfg, seed=0, group=group)
        g = torch.Generator(device="cuda").manual_seed(5)
        ids = torch.randint(0, 50257, (2 * dp, 256), device="cuda", generator=g)
        ids = ids[2 * dpi:2 * dpi + 2].contiguous()  # this group's sequences
        got = tp.forward(ids)
        torch.cuda.synchronize()
        status = tp.status()
        full = gpt2.GPT2(cfg, seed=0)
        v0, v1 = tp.shard.vocab
        one_gpu = full.forward(ids)[..., v0:v1]
        ref = full.reference_forward(ids)[..., v0:v1]
        torch.cuda.synchronize()
        diff = (got - ref).double()
        queue.put((rank, status, float(diff.abs().max() / ref.abs().max()),
                   float(diff.norm() / ref.double().norm()),
                   float((got - one_gpu).abs().max() / one_gpu.abs().max())))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,tp", [(2, 0), (4, 2), (8, 0)])
def test_tensor_parallel_forward(world, tp):
    if not torch.cuda.is_available():
        pytest.fail("a GPU test ran without a CUDA device")
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = torch.multiprocessing.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, queue, tp)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        assert p.exitcode == 0
    for _ in range(world):
        rank, status, worst, norm, vs_one = queue.get(timeout=10)
        assert status == 0, rank
        # logits, tensor-relative (2e-2, the bf16 GEMM paths' tolerance)
        assert worst <= 2e-2 and norm <= 2e-2, (rank, worst, norm)
        # against one GPU: the same kernels, partial products summed in another order
        assert vs_one <= 1e-2, (rank, vs_one)
