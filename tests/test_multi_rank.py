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


# ---------------------------------------------------------------- GPT-2 tensor parallel

def _tp_block_rank(rank: int, world: int, port: int, queue, tp: int = 0) -> None:
    """One block of the TP forward in float32 torch on a gloo rank, with the weights this rank
    holds (ppy_b200.gpt2_tp.shard_block) and the reduction the GPU path makes: rank 0 of the
    group adds its partial product, the bias and the residual, the others their partial
    product, then an all-reduce (sum) over the group. With tp < world the ranks form groups
    of tp (ppy_b200.gpt2_tp.hybrid_groups), each with its share of the batch."""
    import torch.distributed as dist
    import torch.nn.functional as F

    sys.path.insert(0, str(REPO))
    from ppy_b200.gpt2 import Config
    from ppy_b200.gpt2_tp import hybrid_groups, hybrid_layout, shard_block, shard_ranges

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    cfg = Config(layers=1, width=256, heads=4, vocab=1000, context=128)
    c, d, heads = cfg.width, cfg.head_dim, cfg.heads
    g = torch.Generator().manual_seed(11)
    blk = {"ln1_g": 1 + 0.1 * torch.randn(c, generator=g), "ln1_b": 0.1 * torch.randn(c, generator=g),
           "w_qkv": 0.05 * torch.randn(3 * c, c, generator=g), "b_qkv": 0.1 * torch.randn(3 * c, generator=g),
           "w_o": 0.05 * torch.randn(c, c, generator=g), "b_o": 0.1 * torch.randn(c, generator=g),
           "ln2_g": 1 + 0.1 * torch.randn(c, generator=g), "ln2_b": 0.1 * torch.randn(c, generator=g),
           "w_fc": 0.05 * torch.randn(4 * c, c, generator=g), "b_fc": 0.1 * torch.randn(4 * c, generator=g),
           "w_proj": 0.05 * torch.randn(c, 4 * c, generator=g), "b_proj": 0.1 * torch.randn(c, generator=g)}
    dp, tp = hybrid_layout(world, cfg, tp)
    group, dpi = hybrid_groups(tp)
    batch, length = 4 // dp, 64
    x0 = torch.randn(4, length, c, generator=g)[dpi * batch:(dpi + 1) * batch]

    def attention(qkv, nh):
        q, k, v = qkv.split(nh * d, dim=-1)
        shape = lambda t: t.reshape(batch, length, nh, d).transpose(1, 2)  # noqa: E731
        a = F.scaled_dot_product_attention(shape(q), shape(k), shape(v), is_causal=True)
        return a.transpose(1, 2).reshape(batch, length, nh * d)

    # the whole block
    x = x0.clone()
    hh = F.layer_norm(x, (c,), blk["ln1_g"], blk["ln1_b"], 1e-5)
    x = x + F.linear(attention(F.linear(hh, blk["w_qkv"], blk["b_qkv"]), heads), blk["w_o"], blk["b_o"])
    n = F.layer_norm(x, (c,), blk["ln2_g"], blk["ln2_b"], 1e-5)
    x = x + F.linear(F.gelu(F.linear(n, blk["w_fc"], blk["b_fc"]), approximate="tanh"),
                     blk["w_proj"], blk["b_proj"])
    whole = x

    # this rank's share
    shard = shard_ranges(cfg, dist.get_rank(group), tp)
    assert shard.rank == rank % tp
    mine = shard_block(blk, cfg, shard)
    nh = shard.heads[1] - shard.heads[0]

    def row_parallel(a, w, b, x):
        y = x + F.linear(a, w, b) if shard.rank == 0 else F.linear(a, w)
        dist.all_reduce(y, group=group)
        return y

    x = x0.clone()
    hh = F.layer_norm(x, (c,), mine["ln1_g"], mine["ln1_b"], 1e-5)
    x = row_parallel(attention(F.linear(hh, mine["w_qkv"], mine["b_qkv"]), nh), mine["w_o"], mine["b_o"], x)
    n = F.layer_norm(x, (c,), mine["ln2_g"], mine["ln2_b"], 1e-5)
    x = row_parallel(F.gelu(F.linear(n, mine["w_fc"], mine["b_fc"]), approximate="tanh"),
                     mine["w_proj"], mine["b_proj"], x)
    queue.put((rank, float((x - whole).abs().max()), float(whole.abs().max())))
    dist.destroy_process_group()


@pytest.mark.parametrize("world,tp", [(2, 0), (4, 0), (4, 2)])
def test_tensor_parallel_block_equals_the_whole_block(world, tp):
    """Whole tensor-parallel groups, and 4 ranks as 2 data-parallel groups of 2 (the layout 8
    GPUs take as 2 groups of 4)."""
    ctx = torch.multiprocessing.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_tp_block_rank, args=(r, world, port, queue, tp))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
        assert p.exitcode == 0
    for _ in range(world):
        rank, err, scale = queue.get(timeout=10)
        assert err <= 1e-5 * scale, (rank, err, scale)


def test_tensor_parallel_shards_tile_the_model():
    sys.path.insert(0, str(REPO))
    from ppy_b200.gpt2 import GPT2_124M
    from ppy_b200.gpt2_tp import shard_ranges

    for size in (1, 2, 4):
        shards = [shard_ranges(GPT2_124M, r, size) for r in range(size)]
        for key, total in (("heads", 12), ("hidden", 3072), ("vocab", 50257)):
            spans = [getattr(s, key) for s in shards]
            assert spans[0][0] == 0 and spans[-1][1] == total
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
    with pytest.raises(ValueError):
        shard_ranges(GPT2_124M, 0, 8)  # 96-wide slices are not whole 64-wide K steps


def test_hybrid_layouts():
    sys.path.insert(0, str(REPO))
    from ppy_b200.gpt2 import GPT2_124M
    from ppy_b200.gpt2_tp import hybrid_layout

    assert [hybrid_layout(w, GPT2_124M) for w in (1, 2, 4, 8)] == [(1, 1), (1, 2), (1, 4), (2, 4)]
    assert hybrid_layout(8, GPT2_124M, tp=2) == (4, 2)
    assert hybrid_layout(6, GPT2_124M) == (1, 6)  # 2 heads and 128-wide slices per rank
    assert hybrid_layout(16, GPT2_124M) == (4, 4)
    for world, tp in ((8, 8), (6, 4), (4, 3)):
        with pytest.raises(ValueError):
            hybrid_layout(world, GPT2_124M, tp)
