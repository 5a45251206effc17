"""Benchmark of the B200 path: one JSON line per run.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload gelu|rows|collatz]
                    [--impl b200|reference]

A step is one pass of the hot path over one batch of seeded synthetic input:

* gelu    -- y = gelu_tanh(a*b + c) over three fp32 vectors of 2^24 elements (uniform
             [-4, 4], seed 0): the fused elementwise group, through the module the b200
             backend builds from tests/golden/gelu.ppyir. Metric: GB/s of algorithmic
             traffic (16 B per element).
* rows    -- softmax then layernorm over each row of an fp32 [65536, 1024] matrix
             (N(0,1), seed 0; gamma ~ N(1, .02), beta ~ N(0, .02)): the row group built
             from tests/golden/rows.ppyir. Metric: GB/s (8 B per element + gamma, beta).
* collatz -- the step counts of every start in [1, 2^26) summed and maxed: the
             parallel.reduce kernels built from tests/golden/collatz.ppyir. Metric:
             Collatz steps per second.

`value` is device-timed (CUDA events, inputs resident in HBM); `e2e` is the same metric
through the host-memory C-ABI entry point (pinned host buffers, H2D and D2H inside the
timed region). With --gpus N under torchrun each rank runs its own batch (weak scaling)
or its slice of the Collatz range (strong), the time is the max over ranks.
`--impl reference` times the oracle's C restatement of the reference's CPU loops on the
host cores instead (rank 0 only).
"""

from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))
PREBUILT = REPO / "ppy_b200" / "prebuilt"

GELU_N = 1 << 24
ROWS, COLS = 65536, 1024
COLLATZ_HI = 1 << 26


def _args():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=200)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--workload", default="gelu",
                   choices=["gelu", "rows", "collatz", "gemm", "gpt2", "gpt2_tp"])
    p.add_argument("--impl", default="b200", choices=["b200", "reference"])
    p.add_argument("--tp", type=int, default=0,
                   help="gpt2_tp: ranks per tensor-parallel group (0: the widest that fits)")
    p.add_argument("--exchange", default="nvlink", choices=["nvlink", "nccl"],
                   help="gpt2_tp: the row-parallel sum fused into the GEMM over NVLink, or "
                        "an NCCL all-reduce after it")
    p.add_argument("--cpu-seconds", type=float, default=10.0,
                   help="CPU-baseline sample length (seconds of host work)")
    return p.parse_args()


# ---------------------------------------------------------------- distributed plumbing


def shard_range(lo: int, hi: int, world: int, rank: int) -> tuple[int, int]:
    """Rank `rank`'s contiguous slice of [lo, hi): equal spans, the last one shorter."""
    span = (hi - lo + world - 1) // world
    start = min(hi, lo + rank * span)
    return start, min(hi, start + span)


def shard_batch(batch: int, world: int, rank: int) -> tuple[int, int]:
    """Rank `rank`'s sequences [start, stop) of a batch that splits evenly."""
    if batch % world:
        raise SystemExit(f"a batch of {batch} does not split over {world} GPUs")
    per = batch // world
    return rank * per, (rank + 1) * per


class Dist:
    def __init__(self, gpus: int) -> None:
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        self.gpus = gpus
        self.pg = None

    def start(self, backend: str) -> None:
        if self.world > 1:
            import datetime

            import torch.distributed as dist

            dist.init_process_group(backend, timeout=datetime.timedelta(seconds=120))
            self.pg = dist

    def barrier(self) -> None:
        if self.pg is not None:
            if self.pg.get_backend() == "nccl":
                import torch

                self.pg.barrier(device_ids=[self.local])
                torch.cuda.synchronize()
            else:
                self.pg.barrier()

    def max(self, value: float) -> float:
        if self.pg is None:
            return value
        import torch

        device = "cuda" if self.pg.get_backend() == "nccl" else "cpu"
        t = torch.tensor([value], dtype=torch.float64, device=device)
        self.pg.all_reduce(t, op=self.pg.ReduceOp.MAX)
        return float(t.item())

    def sum_i64(self, values: list[int], op: str = "sum") -> list[int]:
        if self.pg is None:
            return values
        import torch

        device = "cuda" if self.pg.get_backend() == "nccl" else "cpu"
        t = torch.tensor(values, dtype=torch.int64, device=device)
        self.pg.all_reduce(t, op=self.pg.ReduceOp.SUM if op == "sum" else self.pg.ReduceOp.MAX)
        return [int(v) for v in t.tolist()]

    def stop(self) -> None:
        if self.pg is not None:
            self.pg.destroy_process_group()


# ---------------------------------------------------------------- clocks


class Clocks:
    """nvidia-smi samples every 20 ms (SM clock, throttle reasons) around the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int) -> None:
        self.device = device
        self.samples: list[tuple[float, list[str]]] = []
        self.window: tuple[float, float] | None = None
        self.process = None
        self._thread = threading.Thread(target=self._read, daemon=True)

    def _read(self) -> None:
        for line in self.process.stdout:
            fields = [x.strip() for x in line.split(",")]
            if len(fields) >= 9:
                self.samples.append((time.perf_counter(), fields))

    def start(self) -> None:
        try:
            self.process = subprocess.Popen(
                ["nvidia-smi", f"--id={self.device}", f"--query-gpu={self.QUERY}",
                 "--format=csv,noheader,nounits", "-lms", "20"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self._thread.start()
        except OSError:
            self.process = None

    def mark(self, begin: float, end: float) -> None:
        self.window = (begin, end)

    def stop(self) -> dict:
        if self.process is not None:
            time.sleep(0.05)
            self.process.terminate()
            try:
                self.process.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.process.kill()
            self._thread.join(timeout=5)
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        inside = [s for t, s in self.samples
                  if self.window and self.window[0] - 0.02 <= t <= self.window[1] + 0.02]
        chosen = inside or [s for _, s in self.samples]

        def number(text):
            try:
                return float(text)
            except ValueError:
                return None

        sm = sorted(v for v in (number(s[1]) for s in chosen) if v is not None)
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for s in chosen:
            for name, flag in zip(names, s[5:9]):
                if flag.lower().startswith("active"):
                    reasons.add(name)
        return {"sm_mhz": sm[len(sm) // 2] if sm else None,
                "sm_max_mhz": number(chosen[0][2]), "reasons": sorted(reasons),
                "samples": len(chosen), "samples_in_timed_region": len(inside)}


def peaks() -> dict:
    path = REPO / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        return {"hbm_gbs": data["hbm_gbs"], "source": "measured"}
    return {"hbm_gbs": 6650.0, "source": "fallback"}


def traffic(kernel: str) -> float | None:
    """DRAM bytes per launch of `kernel` from the committed ncu summary, if any."""
    path = REPO / "profiles" / "traffic.json"
    if not path.exists():
        return None
    data = json.loads(path.read_text())
    entry = data.get(kernel)
    return float(entry["bytes_per_launch"]) if entry else None


# ---------------------------------------------------------------- workloads


class Workload:
    metric = ""
    unit = ""
    dtype = ""
    kernel = ""
    scaling = "weak"

    def __init__(self, dist: Dist) -> None:
        self.dist = dist


class Gelu(Workload):
    metric = "fused-group GB/s: y = gelu_tanh(a*b + c), fp32, 2^24 elements"
    unit = "GB/s"
    dtype = "f32"
    kernel = "gelu_chain_k0_v"
    bytes_per_step = 16 * GELU_N

    def inputs(self):
        rng = np.random.default_rng(0 + self.dist.rank)
        self.host = [rng.uniform(-4, 4, GELU_N).astype(np.float32) for _ in range(3)]

    def config(self):
        return {"workload": "gelu_chain_f32", "elements": GELU_N, "seed": 0,
                "bytes_per_step": self.bytes_per_step,
                "l2": "inputs larger than L2 (201 MB read per step), no flush"}

    def setup_device(self, runtime, torch):
        self.module = runtime.load(PREBUILT / "gelu" / "gelu.json")
        self.dev = [torch.from_numpy(x).cuda() for x in self.host]
        self.out = torch.empty_like(self.dev[0])
        self.pinned = [torch.from_numpy(x).pin_memory() for x in self.host]
        self.pinned_out = torch.empty(GELU_N, dtype=torch.float32).pin_memory()

    def step_device(self):
        return self.module.device.gelu_chain(*self.dev, self.out).status

    def step_host(self):
        return self.module.gelu_chain(*self.pinned, self.pinned_out).status

    def h2d_d2h(self):
        return 12 * GELU_N, 4 * GELU_N

    def cpu_step(self, threads: int, oracle):
        # a bounded sample of the batch: the first 2^22 elements
        n = 1 << 22
        oracle.gelu_chain(self.host[0][:n], self.host[1][:n], self.host[2][:n], threads=threads)
        return 16 * n

    def check(self, oracle):
        sample = slice(0, 1 << 16)
        expected = oracle.gelu_chain(self.host[0][sample].copy(), self.host[1][sample].copy(),
                                     self.host[2][sample].copy())
        got = self.out[: 1 << 16].cpu().numpy()
        scale = np.maximum(np.abs(expected), 1.0)
        return float(np.max(np.abs(got - expected) / scale))


class Rows(Workload):
    metric = "fused-group GB/s: row softmax -> layernorm, fp32 [65536, 1024]"
    unit = "GB/s"
    dtype = "f32"
    kernel = "softmax_layernorm_k0"
    bytes_per_step = 2 * 4 * ROWS * COLS + 2 * 4 * COLS

    def inputs(self):
        rng = np.random.default_rng(0 + self.dist.rank)
        self.x = rng.standard_normal((ROWS, COLS), dtype=np.float32)
        self.gamma = (1 + 0.02 * rng.standard_normal(COLS)).astype(np.float32)
        self.beta = (0.02 * rng.standard_normal(COLS)).astype(np.float32)

    def config(self):
        return {"workload": "softmax_layernorm_rows_f32", "rows": ROWS, "cols": COLS, "seed": 0,
                "bytes_per_step": self.bytes_per_step,
                "l2": "inputs larger than L2 (268 MB read per step), no flush"}

    def setup_device(self, runtime, torch):
        self.module = runtime.load(PREBUILT / "rows" / "rows.json")
        self.dx = torch.from_numpy(self.x).cuda()
        self.dg = torch.from_numpy(self.gamma).cuda()
        self.db = torch.from_numpy(self.beta).cuda()
        self.out = torch.empty_like(self.dx)
        self.px = torch.from_numpy(self.x).pin_memory()
        self.pout = torch.empty_like(self.px).pin_memory()

    def step_device(self):
        return self.module.device.softmax_layernorm(self.dx, self.dg, self.db, self.out).status

    def step_host(self):
        return self.module.softmax_layernorm(self.px.view(-1), torch_from(self.gamma),
                                             torch_from(self.beta), self.pout.view(-1)).status

    def h2d_d2h(self):
        return 4 * ROWS * COLS + 8 * COLS, 4 * ROWS * COLS

    def cpu_step(self, threads: int, oracle):
        rows = 4096
        oracle.softmax_layernorm(self.x[:rows], self.gamma, self.beta, threads=threads)
        return 2 * 4 * rows * COLS

    def check(self, oracle):
        expected = oracle.softmax_layernorm(self.x[:256].copy(), self.gamma, self.beta)
        got = self.out[:256].cpu().numpy()
        return float(np.max(np.abs(got - expected) / np.maximum(np.abs(expected), 1.0)))


def torch_from(array):
    import torch

    return torch.from_numpy(array)


class Collatz(Workload):
    metric = "Collatz steps/s: parallel.range(1, 2^26) int64 sum and max of step counts"
    unit = "steps/s"
    dtype = "int64"
    kernel = "par_collatz_collatz_sum_0_part"
    scaling = "strong"

    def inputs(self):
        self.lo, self.hi = shard_range(1, COLLATZ_HI, self.dist.world, self.dist.rank)
        self.total_steps = None

    def config(self):
        return {"workload": "collatz_parallel_range", "range": [1, COLLATZ_HI],
                "rank_range": [self.lo, self.hi], "l2": "no data: integer-issue bound"}

    def setup_device(self, runtime, torch):
        self.module = runtime.load(PREBUILT / "collatz" / "collatz.json")

    def step_device(self):
        status, self.sum = self.module.device.collatz_collatz_sum(self.lo, self.hi)
        status2, self.best = self.module.device.collatz_collatz_max(self.lo, self.hi)
        return status or status2

    step_host = step_device

    def h2d_d2h(self):
        return 32, 16  # (lo, hi) twice in, (sum, max) out

    def cpu_step(self, threads: int, oracle):
        hi = min(self.hi, self.lo + (1 << 22))
        status, total, _best = oracle.collatz(self.lo, hi, threads)
        return total

    def check(self, oracle):
        return 0.0


class Gemm(Workload):
    metric = "matmul TFLOP/s: C = A @ B + bias, bf16 A/B, f32 accumulate and C, 8192^3"
    unit = "TFLOP/s"
    dtype = "bf16"
    kernel = "matmul_bf16_pair_kernel"  # K = 8192: CTA pairs
    M = N = K = 8192
    flops = 2 * 8192 ** 3

    def inputs(self):
        import torch

        g = torch.Generator().manual_seed(0 + self.dist.rank)
        k = self.K
        self.a = (torch.randn(self.M, k, generator=g) / k ** 0.5).to(torch.bfloat16)
        self.b = (torch.randn(k, self.N, generator=g) / k ** 0.5).to(torch.bfloat16)
        self.bias = 0.02 * torch.randn(self.N, generator=g)

    def config(self):
        return {"workload": "matmul_bias_bf16", "m": self.M, "n": self.N, "k": self.K,
                "seed": 0, "flops_per_step": self.flops,
                "path": "tensor.matmul of tensor.convert(bf16) + bias through the built module: "
                        "B [K,N] transposed to K-major, then the tcgen05 kernel",
                "l2": "operands 256 MB > L2, no flush"}

    def setup_device(self, runtime, torch):
        self.module = runtime.load(PREBUILT / "matmul_bf16_8192" / "matmul_bf16_8192.json")
        self.da, self.db, self.dbias = self.a.cuda(), self.b.cuda(), self.bias.cuda()
        self.out = torch.empty(self.M, self.N, device="cuda")
        self.pa, self.pb = self.a.pin_memory(), self.b.pin_memory()
        self.pbias = self.bias.pin_memory()
        self.pout = torch.empty(self.M, self.N).pin_memory()
        self.dbt = self.db.t().contiguous()
        import ctypes

        self.lib = runtime.library()
        self.lib.ppyb200_matmul_bf16_kmajor.argtypes = [ctypes.c_void_p] * 4 + [ctypes.c_int64] * 3

    def step_device(self):
        return self.module.device.matmul_bias_bf16(self.da, self.db, self.dbias, self.out).status

    def step_host(self):
        import torch

        return self.module.matmul_bias_bf16(self.pa.view(torch.int16), self.pb.view(torch.int16),
                                            self.pbias, self.pout).status

    def kernel_step(self):
        """The tcgen05 kernel alone (B already K-major): the roofline's launch."""
        return self.lib.ppyb200_matmul_bf16_kmajor(self.da.data_ptr(), self.dbt.data_ptr(),
                                                   self.dbias.data_ptr(), self.out.data_ptr(),
                                                   self.M, self.N, self.K)

    def h2d_d2h(self):
        return 2 * 2 * self.M * self.K + 4 * self.N, 4 * self.M * self.N

    def cpu_step(self, threads: int, oracle):
        # NumPy f32 BLAS on the bf16-rounded values (the CPython reference of the path),
        # over a bounded sample: the first 512 rows of A
        rows = 512
        a = self.a[:rows].float().numpy()
        b = self.b.float().numpy()
        _ = a @ b + self.bias.numpy()
        return 2 * rows * self.N * self.K

    def check(self, oracle):
        import torch

        rows = torch.tensor([0, 4095, 8191])
        ref = self.a[rows].double() @ self.b.double() + self.bias.double()
        got = self.out[rows.cuda()].cpu().double()
        scale = torch.maximum(ref.abs(), ref.pow(2).mean().sqrt())
        return float(((got - ref).abs() / scale).max())


class Gpt2(Workload):
    metric = "GPT-2-124M forward tokens/s: batch 32 x 1024, logits out"
    unit = "tokens/s"
    dtype = "bf16"
    kernel = "gpt2_forward"
    scaling = "strong"
    BATCH, LENGTH = 32, 1024

    def inputs(self):
        import torch

        start, stop = shard_batch(self.BATCH, self.dist.world, self.dist.rank)
        g = torch.Generator().manual_seed(0)
        ids = torch.randint(0, 50257, (self.BATCH, self.LENGTH), generator=g)
        self.ids = ids[start:stop].contiguous()

    def config(self):
        return {"workload": "gpt2_124m_forward", "batch": self.BATCH, "seq_len": self.LENGTH,
                "layers": 12, "width": 768, "heads": 12, "vocab": 50257,
                "parallelism": f"dp{self.dist.world}", "weights": "N(0, 0.02) seed 0, bf16",
                "l2": "weights 250 MB + activations > L2, no flush"}

    def setup_device(self, runtime, torch):
        from ppy_b200 import gpt2

        self.model = gpt2.GPT2(gpt2.GPT2_124M, seed=0)
        self.gpt2 = gpt2
        self.dids = self.ids.cuda()
        self.pids = self.ids.pin_memory()
        b = self.ids.shape[0]
        self.logits = self.model.new_logits(b, self.LENGTH)  # rows on 128-byte lines
        self.last = torch.empty(b, 50257).pin_memory()

    def step_device(self):
        self.model.forward(self.dids, self.logits)
        return 0

    def step_host(self):
        # e2e: ids from pinned host memory in, the last position's logits out (what the
        # next-token step reads)
        self.dids.copy_(self.pids, non_blocking=True)
        self.model.forward(self.dids, self.logits)
        self.last.copy_(self.logits[:, -1], non_blocking=True)
        return 0

    def h2d_d2h(self):
        b = self.ids.shape[0]
        return 8 * b * self.LENGTH, 4 * b * 50257

    def cpu_step(self, threads: int, oracle):
        # the reference's GPT-2 path is torch ATen: its CPU forward, one sequence of 1024,
        # f32 weights (the bf16-rounded values)
        import torch

        if not hasattr(self, "cpu_model"):
            self.cpu_model = _cpu_reference_model()
        torch.set_num_threads(threads)
        with torch.no_grad():
            self.cpu_model(self.ids[:1])
        return float(self.LENGTH)

    def check(self, oracle):
        import torch

        ids = self.dids[:1, :256]
        got = self.model.forward(ids)
        ref = self.model.reference_forward(ids)
        torch.cuda.synchronize()
        return float((got - ref).abs().max() / ref.abs().max())


class Gpt2TP(Gpt2):
    """The tensor-parallel variant: the ranks of a group work on the group's sequences with
    12/T heads, 3072/T hidden units and 50257/T logits columns each, two all-reduces of the
    residual stream per block (T in {1, 2, 4}); N ranks form N/T such groups, each with its
    share of the batch (8 GPUs: 2 groups of 4). `--tp` picks T, 0 the widest that fits."""

    metric = "GPT-2-124M forward tokens/s, tensor parallel: batch 32 x 1024, logits out"
    kernel = "gpt2_tp_forward"
    tp = 0
    exchange = "nvlink"

    def inputs(self):
        import torch

        from ppy_b200 import gpt2, gpt2_tp

        self.dp, self.tp = gpt2_tp.hybrid_layout(self.dist.world, gpt2.GPT2_124M, self.tp)
        start, stop = shard_batch(self.BATCH, self.dp, self.dist.rank // self.tp)
        g = torch.Generator().manual_seed(0)
        ids = torch.randint(0, 50257, (self.BATCH, self.LENGTH), generator=g)
        self.ids = ids[start:stop].contiguous()

    def config(self):
        cfg = super().config()
        tokens = self.ids.numel()
        if self.exchange == "nvlink":
            exchange = (f"fused: each row-parallel GEMM's epilogue stores its f32 [{tokens}, "
                        f"768] partial into every rank of its group of {self.tp} over NVLink, "
                        "then a flag per rank and an in-order sum; 2 per block")
        else:
            exchange = (f"2 NCCL all-reduces (sum, f32 [{tokens}, 768]) per block inside "
                        f"each group of {self.tp}")
        cfg.update(workload="gpt2_124m_forward_tp",
                   parallelism=f"tp{self.tp}" if self.dp == 1 else f"dp{self.dp}xtp{self.tp}",
                   exchange=exchange)
        return cfg

    def setup_device(self, runtime, torch):
        from ppy_b200 import gpt2, gpt2_tp

        group = None
        if self.dist.world > 1:
            group, _ = gpt2_tp.hybrid_groups(self.tp)
        self.model = gpt2_tp.GPT2TensorParallel(gpt2.GPT2_124M, seed=0, group=group,
                                                exchange=self.exchange)
        self.gpt2 = gpt2
        self.dids = self.ids.cuda()
        self.pids = self.ids.pin_memory()
        v0, v1 = self.model.shard.vocab
        b = self.ids.shape[0]
        self.logits = self.model.new_logits(b, self.LENGTH)  # rows on 128-byte lines
        self.last = torch.empty(b, v1 - v0).pin_memory()

    def h2d_d2h(self):
        v0, v1 = self.model.shard.vocab
        b = self.ids.shape[0]
        return 8 * b * self.LENGTH, 4 * b * (v1 - v0)

    def check(self, oracle):
        import torch

        full = self.gpt2.GPT2(self.gpt2.GPT2_124M, seed=0)
        ids = self.dids[:1, :256]
        got = self.model.forward(ids)
        v0, v1 = self.model.shard.vocab
        ref = full.reference_forward(ids)[..., v0:v1]
        torch.cuda.synchronize()
        return float((got - ref).abs().max() / ref.abs().max())


def _cpu_reference_model():
    """The GPT-2 forward of examples/46_gpt2/gpt2.ppy:18-57 (torch ATen ops) on the CPU, the
    same shapes and init, f32."""
    import torch
    import torch.nn.functional as F

    g = torch.Generator().manual_seed(0)
    c, v, layers, heads = 768, 50257, 12, 12

    def normal(*shape):
        return (0.02 * torch.randn(*shape, generator=g)).to(torch.bfloat16).float()

    wte, wpe = normal(v, c), normal(1024, c)
    blocks = [(normal(3 * c, c), normal(c, c), normal(4 * c, c), normal(c, 4 * c))
              for _ in range(layers)]
    ones, zeros = torch.ones(c), torch.zeros(c)

    def forward(ids):
        b, n = ids.shape
        x = wte[ids] + wpe[:n]
        for wqkv, wo, wfc, wproj in blocks:
            h = F.layer_norm(x, (c,), ones, zeros, 1e-5)
            q, k, vv = F.linear(h, wqkv).split(c, dim=-1)
            shape = lambda t: t.reshape(b, n, heads, c // heads).transpose(1, 2)  # noqa: E731
            a = F.scaled_dot_product_attention(shape(q), shape(k), shape(vv), is_causal=True)
            x = x + F.linear(a.transpose(1, 2).reshape(b, n, c), wo)
            f = F.gelu(F.linear(F.layer_norm(x, (c,), ones, zeros, 1e-5), wfc), approximate="tanh")
            x = x + F.linear(f, wproj)
        return F.layer_norm(x, (c,), ones, zeros, 1e-5) @ wte.t()

    return forward


WORKLOADS = {"gelu": Gelu, "rows": Rows, "collatz": Collatz, "gemm": Gemm, "gpt2": Gpt2,
             "gpt2_tp": Gpt2TP}


def units_per_step(w: Workload) -> float:
    if isinstance(w, Gemm):
        return float(w.flops)
    if isinstance(w, Gpt2):
        return float(w.ids.numel())
    if isinstance(w, Collatz):
        if w.total_steps is None:
            w.total_steps = w.sum
        return float(w.total_steps)
    return float(w.bytes_per_step)


def to_metric(w: Workload, units: float, seconds: float) -> float:
    if w.unit == "GB/s":
        return units / seconds / 1e9
    if w.unit == "TFLOP/s":
        return units / seconds / 1e12
    return units / seconds


def cpu_baseline(w: Workload, seconds: float) -> dict:
    import oracle

    threads = oracle.threads_available()
    done = 0.0
    start = time.perf_counter()
    steps = 0
    while True:
        done += w.cpu_step(threads, oracle)
        steps += 1
        elapsed = time.perf_counter() - start
        if elapsed >= seconds:
            break
    sample = {"gpt2": "torch CPU forward (f32) of the first sequence (1 x 1024), repeated",
              "gpt2_tp": "torch CPU forward (f32) of the first sequence (1 x 1024), repeated",
              "gemm": "NumPy f32 BLAS on the first 512 rows of A, repeated",
              "gelu": "first 2^22 elements of the batch, repeated",
              "rows": "first 4096 rows of the batch, repeated",
              "collatz": "starts [lo, lo + 2^22) of the range, repeated"}[
        next(k for k, v in WORKLOADS.items() if isinstance(w, v))]
    return {"value": to_metric(w, done, elapsed), "unit": w.unit, "cores": threads,
            "kind": "port", "sample": f"{sample}; {steps} passes in {elapsed:.1f} s"}


def run_reference(args, dist: Dist) -> None:
    dist.start("gloo")
    if dist.rank != 0:
        dist.stop()
        return
    w = WORKLOADS[args.workload](dist)
    w.dist.world = 1
    w.inputs()
    import oracle

    threads = oracle.threads_available()
    for _ in range(args.warmup):
        w.cpu_step(threads, oracle)
    units = 0.0
    start = time.perf_counter()
    for _ in range(args.steps):
        units += w.cpu_step(threads, oracle)
    elapsed = time.perf_counter() - start
    value = to_metric(w, units, elapsed)
    line = {"metric": w.metric, "value": value, "unit": w.unit, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": elapsed / max(args.steps, 1) * 1e3, "higher_is_better": True,
            "scaling": w.scaling, "vs_baseline": None, "dtype": w.dtype, "data": "synthetic",
            "config": w.config(), "impl": "reference",
            "cpu_baseline": {"value": value, "unit": w.unit, "cores": threads, "kind": "port",
                             "sample": "one bounded sample of the batch per step (oracle C "
                                       "restatement of the reference's CPU loops, OpenMP)"},
            "e2e": {"value": value, "unit": w.unit, "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    dist.stop()


def run_b200(args, dist: Dist) -> None:
    import torch

    from ppy_b200 import runtime

    torch.cuda.set_device(dist.local)
    dist.start("nccl")
    runtime.init(dist.local)
    # one stream for everything: the module's launches, copies and the timing events
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    runtime.set_stream(stream)
    w = WORKLOADS[args.workload](dist)
    w.tp = args.tp
    w.exchange = args.exchange
    w.inputs()
    w.setup_device(runtime, torch)
    clocks = Clocks(dist.local)
    clocks.start()
    for _ in range(max(args.warmup, 3)):
        assert w.step_device() == 0
        assert w.step_host() == 0
    torch.cuda.synchronize()
    # device-resident timing: K steps back to back between one event pair
    start_event = torch.cuda.Event(enable_timing=True)
    end_event = torch.cuda.Event(enable_timing=True)
    launches0 = runtime.launches()
    dist.barrier()
    torch.cuda.synchronize()
    begin = time.perf_counter()
    start_event.record(stream)
    for _ in range(args.steps):
        status = w.step_device()
        if status != 0:
            raise SystemExit(f"step failed with status {status}")
    end_event.record(stream)
    torch.cuda.synchronize()
    dist.barrier()
    end = time.perf_counter()
    clocks.mark(begin, end)
    launches = runtime.launches() - launches0
    total_ms = dist.max(start_event.elapsed_time(end_event))
    # the dominant kernel's own launch duration (for the workloads whose step is more than
    # that one launch, timed alone over the same number of launches)
    if hasattr(w, "kernel_step"):
        k0 = torch.cuda.Event(enable_timing=True)
        k1 = torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        k0.record(stream)
        for _ in range(args.steps):
            if w.kernel_step() != 0:
                raise SystemExit("kernel step failed")
        k1.record(stream)
        torch.cuda.synchronize()
        step_ms = [k0.elapsed_time(k1) / args.steps]
    else:
        step_ms = [total_ms / args.steps]
    units = units_per_step(w)
    units_all = units * (dist.world if w.scaling == "weak" else 1)
    if isinstance(w, Collatz):
        sums = dist.sum_i64([w.sum])
        units_all = float(sums[0])
    if isinstance(w, Gpt2TP):
        units_all = float(units) * w.dp  # the ranks of a group share their tokens
    elif isinstance(w, Gpt2):
        units_all = float(dist.sum_i64([int(units)])[0])
    value = to_metric(w, units_all * args.steps, total_ms / 1e3)
    kernel_ms = float(np.mean(step_ms))
    # end to end through the host-memory entry point (pinned host buffers)
    e_start = torch.cuda.Event(enable_timing=True)
    e_end = torch.cuda.Event(enable_timing=True)
    dist.barrier()
    torch.cuda.synchronize()
    launches1 = runtime.launches()
    e_start.record(stream)
    for _ in range(args.steps):
        if w.step_host() != 0:
            raise SystemExit("host-memory step failed")
    e_end.record(stream)
    torch.cuda.synchronize()
    dist.barrier()
    launches += runtime.launches() - launches1
    e2e_ms = dist.max(e_start.elapsed_time(e_end))
    e2e = to_metric(w, units_all * args.steps, e2e_ms / 1e3)
    clock_info = clocks.stop()
    import oracle

    error = w.check(oracle)
    if dist.rank == 0:
        pk = peaks()
        h2d, d2h = w.h2d_d2h()
        line = {"metric": w.metric, "value": value, "unit": w.unit, "n_gpus": dist.world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": total_ms / args.steps,
                "higher_is_better": True, "scaling": w.scaling, "vs_baseline": None,
                "dtype": w.dtype, "data": "synthetic (seeded)", "config": w.config(),
                "e2e": {"value": e2e, "unit": w.unit, "h2d_bytes_per_step": h2d,
                        "d2h_bytes_per_step": d2h},
                "gpu_launches": int(launches), "clocks": clock_info,
                "max_rel_error_vs_oracle": error}
        if w.unit == "TFLOP/s":
            pk_t = json.loads((REPO / "MEASURED_PEAKS.json").read_text())["bf16_tflops"] if (
                REPO / "MEASURED_PEAKS.json").exists() else 1590.0
            achieved = w.flops / (kernel_ms / 1e3) / 1e12
            line["roofline"] = {"bound": "tensor", "achieved": achieved, "peak": pk_t,
                                "unit": "TFLOP/s", "frac": achieved / pk_t,
                                "traffic": traffic(w.kernel), "peak_source": pk["source"],
                                "kernel": w.kernel, "kernel_ms": kernel_ms}
        elif w.unit == "GB/s":
            achieved = w.bytes_per_step / (kernel_ms / 1e3) / 1e9
            line["roofline"] = {"bound": "hbm", "achieved": achieved, "peak": pk["hbm_gbs"],
                                "unit": "GB/s", "frac": achieved / pk["hbm_gbs"],
                                "traffic": traffic(w.kernel), "peak_source": pk["source"],
                                "kernel": w.kernel, "kernel_ms": kernel_ms}
        elif isinstance(w, Gpt2TP):
            pk_t = json.loads((REPO / "MEASURED_PEAKS.json").read_text())["bf16_tflops_sustained"] if (
                REPO / "MEASURED_PEAKS.json").exists() else 1400.0
            per_gpu = w.gpt2.sequence_flops(w.gpt2.GPT2_124M, w.BATCH, w.LENGTH) / dist.world / (
                total_ms / args.steps / 1e3) / 1e12
            line["roofline"] = {"bound": "tensor", "achieved": per_gpu, "peak": pk_t,
                                "unit": "TFLOP/s", "frac": per_gpu / pk_t, "traffic": None,
                                "peak_source": "measured (sustained)", "kernel": w.kernel,
                                "kernel_ms": total_ms / args.steps}
        elif isinstance(w, Gpt2):
            pk_t = json.loads((REPO / "MEASURED_PEAKS.json").read_text())["bf16_tflops_sustained"] if (
                REPO / "MEASURED_PEAKS.json").exists() else 1400.0
            table = w.model.profile(w.dids, w.logits)
            name, (count, ms, flops) = max(table.items(), key=lambda kv: kv[1][1])
            achieved = flops / (ms / 1e3) / 1e12
            forward_tflops = w.gpt2.sequence_flops(w.gpt2.GPT2_124M, w.ids.shape[0],
                                                   w.LENGTH) / (total_ms / args.steps / 1e3) / 1e12
            line["roofline"] = {"bound": "tensor", "achieved": achieved, "peak": pk_t,
                                "unit": "TFLOP/s", "frac": achieved / pk_t, "traffic": None,
                                "peak_source": "measured (sustained)", "kernel": name,
                                "kernel_ms": ms / count,
                                "forward_tflops": forward_tflops,
                                "forward_frac": forward_tflops / pk_t,
                                "breakdown_ms": {k: round(v[1], 3) for k, v in table.items()}}
        else:
            line["roofline"] = {"bound": "int-issue", "achieved": value, "peak": None,
                                "unit": w.unit, "frac": None, "traffic": None,
                                "kernel": w.kernel, "kernel_ms": kernel_ms}
        if dist.world == 1:
            line["cpu_baseline"] = cpu_baseline(w, args.cpu_seconds)
        print(json.dumps(line), flush=True)
    close = getattr(getattr(w, "model", None), "close", None)
    if close is not None:
        close()  # the tensor-parallel exchange buffers: every rank of the group together
    dist.stop()


def main() -> None:
    args = _args()
    dist = Dist(args.gpus)
    if args.impl == "reference":
        run_reference(args, dist)
    else:
        run_b200(args, dist)


if __name__ == "__main__":
    main()
