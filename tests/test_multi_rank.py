"""The multi-GPU host logic on CPU ranks (gloo, world size 2): how bench.py splits the work and
combines it. The Collatz range is the path's only exchange (a sum and a max of two int64);
maps, rows and GPT-2 sequences split with no collective on the data path."""

from __future__ import annotations

import json
import os
import socket
import subprocess
import sys

import pytest

from conftest import REPO

torch = pytest.importorskip("torch")


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_shards_cover_the_range_and_the_batch():
    sys.path.insert(0, str(REPO))
    import bench

    for world in (1, 2, 3, 4, 8):
        spans = [bench.shard_range(1, 1 << 26, world, r) for r in range(world)]
        assert spans[0][0] == 1 and spans[-1][1] == 1 << 26
        assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
    for world in (1, 2, 4, 8):
        parts = [bench.shard_batch(32, world, r) for r in range(world)]
        assert parts[0][0] == 0 and parts[-1][1] == 32
    with pytest.raises(SystemExit):
        bench.shard_batch(32, 3, 0)


def _collatz_rank(rank: int, world: int, port: int, queue) -> None:
    import torch.distributed as dist

    sys.path.insert(0, str(REPO))
    import bench
    import oracle

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    lo, hi = bench.shard_range(1, 1 << 18, world, rank)
    status, total, best = oracle.collatz(lo, hi, 1)
    t = torch.tensor([total], dtype=torch.int64)
    m = torch.tensor([best], dtype=torch.int64)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    dist.all_reduce(m, op=dist.ReduceOp.MAX)
    if rank == 0:
        queue.put((status, int(t.item()), int(m.item())))
    dist.destroy_process_group()


def test_collatz_split_and_all_reduce_give_the_whole_range():
    import oracle

    ctx = torch.multiprocessing.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_collatz_rank, args=(r, 2, port, queue)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    status, total, best = queue.get(timeout=10)
    assert (status, total, best) == oracle.collatz(1, 1 << 18, 4)


def test_reference_arm_under_torchrun_prints_one_line():
    env = dict(os.environ, OMP_NUM_THREADS="1")
    done = subprocess.run(
        [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
         "--master-addr=127.0.0.1", f"--master-port={_free_port()}", "bench.py", "--impl",
         "reference", "--gpus", "2", "--steps", "1", "--warmup", "0"],
        cwd=REPO, capture_output=True, text=True, env=env, timeout=300, check=False)
    assert done.returncode == 0, done.stderr[-2000:]
    lines = [line for line in done.stdout.splitlines() if line.startswith("{")]
    assert len(lines) == 1
    record = json.loads(lines[0])
    assert record["impl"] == "reference" and record["value"] > 0
    assert record["cpu_baseline"]["kind"] == "port"
