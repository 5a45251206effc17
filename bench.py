"""Benchmark of the B200 path: one JSON line per run.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--impl b200|reference]

A step is one pass of the hot path over one batch of seeded synthetic input. The default
workload is the GPT-2-124M forward, the model half of the headline metric; the fused-group
half (the GELU chain and the softmax->layernorm row group) rides in the same line under
"workloads", each with its own value, e2e, roofline and CPU baseline.

* gpt2     -- GPT-2-124M forward (12 layers, width 768, 12 heads, vocab 50257), N(0, 0.02)
              bf16 weights from seed 0, batch 32 x 1024 token ids (seed 0), f32 logits out;
              data-parallel over the GPUs (32/N sequences each). Metric: tokens/s of the job.
              The forward is captured once into a CUDA graph and replayed each step.
* gpt2_tp  -- the same forward tensor-parallel (groups of --tp GPUs, data-parallel groups).
* gelu     -- y = gelu_tanh(a*b + c) over three fp32 vectors of 2^24 elements (uniform
              [-4, 4], seed 0), the module the backend builds from tests/golden/gelu.ppyir.
              Metric: GB/s of algorithmic traffic (16 B per element).
* rows     -- softmax then layernorm over each row of an fp32 [65536, 1024] matrix (N(0,1),
              seed 0; gamma ~ N(1, .02), beta ~ N(0, .02)), from tests/golden/rows.ppyir.
              Metric: GB/s (8 B per element + gamma, beta).
* collatz  -- the step counts of every start in [1, 2^26) summed and maxed (parallel.reduce
              kernels from tests/golden/collatz.ppyir). Metric: Collatz steps/s.
* gemm     -- C = A @ B + bias, bf16 A and B, f32 accumulate and C, 8192^3. TFLOP/s.
* gemm_f32 -- the fp32-input variant, 4096^3 (three tf32 products on the tensor cores).

`value` is device-timed (CUDA events on the launching stream, inputs resident in HBM, max
over ranks); `e2e` is the same metric through the host-memory path: every step copies its
inputs in from pinned host memory and its whole output back (GPT-2: all logits).
`--impl reference` times the CPU implementation of the path on the host cores instead
(rank 0 only): the oracle's C restatement of the reference's CPU loops, and for GPT-2 the
reference's own path, torch ATen, on the CPU.
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
VOCAB = 50257


def _args():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--workload", default="gpt2",
                   choices=["gpt2", "gpt2_tp", "gelu", "rows", "collatz", "gemm", "gemm_f32"])
    p.add_argument("--extras", default="gelu,rows",
                   help="with the gpt2 workload: the fused-group workloads measured in the same "
                        "run and reported under 'workloads' ('none' for none)")
    p.add_argument("--impl", default="b200", choices=["b200", "reference"])
    p.add_argument("--tp", type=int, default=0,
                   help="gpt2_tp: ranks per tensor-parallel group (0: the widest that fits)")
    p.add_argument("--exchange", default="nvlink", choices=["nvlink", "nccl"],
                   help="gpt2_tp: the row-parallel sum fused into the GEMM over NVLink, or "
                        "an NCCL all-reduce after it")
    p.add_argument("--eager", action="store_true",
                   help="gpt2: launch the forward's kernels one by one instead of replaying a "
                        "CUDA graph")
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
    """nvidia-smi samples every 20 ms (SM clock, throttle reasons); summarised over the
    timed regions marked with `mark`."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int) -> None:
        self.device = device
        self.samples: list[tuple[float, list[str]]] = []
        self.windows: list[tuple[float, float]] = []
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
        self.windows.append((begin, end))

    def stop(self) -> None:
        if self.process is not None:
            time.sleep(0.05)
            self.process.terminate()
            try:
                self.process.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.process.kill()
            self._thread.join(timeout=5)

    def summary(self, windows=None) -> dict:
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        windows = self.windows if windows is None else windows
        inside = [s for t, s in self.samples
                  if any(b - 0.02 <= t <= e + 0.02 for b, e in windows)]
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


def measured_peaks() -> dict:
    """The pool's measured peaks, else the fallback figures (said so in `source`)."""
    path = REPO / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        return {"hbm_gbs": data["hbm_gbs"], "bf16_tflops": data["bf16_tflops"],
                "bf16_tflops_sustained": data["bf16_tflops_sustained"], "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0,
            "source": "fallback"}


def traffic(kernel: str) -> float | None:
    """DRAM bytes per launch of `kernel` from the committed ncu summary, if any."""
    path = REPO / "profiles" / "traffic.json"
    if not path.exists():
        return None
    entry = json.loads(path.read_text()).get(kernel)
    return float(entry["bytes_per_launch"]) if entry else None


# ---------------------------------------------------------------- workloads


class Workload:
    name = ""
    metric = ""
    unit = ""
    dtype = ""
    kernel = ""
    scaling = "weak"
    sample = ""

    def __init__(self, dist: Dist) -> None:
        self.dist = dist
        self.tp = 0
        self.exchange = "nvlink"
        self.eager = False

    def units(self) -> float:
        """Units of the metric one step of this rank processes."""
        return float(self.bytes_per_step)

    def job_units(self) -> float:
        """Units of the metric one step of the whole job processes."""
        return self.units() * (self.dist.world if self.scaling == "weak" else 1)

    def roofline(self, kernel_ms: float, peaks: dict) -> dict:
        achieved = self.bytes_per_step / (kernel_ms / 1e3) / 1e9
        return {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                "frac": achieved / peaks["hbm_gbs"], "traffic": traffic(self.kernel),
                "peak_source": f"{peaks['source']} HBM copy", "kernel": self.kernel,
                "kernel_ms": kernel_ms,
                "algorithmic_bytes_per_launch": self.bytes_per_step}


class Gelu(Workload):
    name = "gelu_chain_f32"
    metric = "fused-group GB/s: y = gelu_tanh(a*b + c), fp32, 2^24 elements"
    unit = "GB/s"
    dtype = "f32"
    kernel = "gelu_chain_k0_v"
    bytes_per_step = 16 * GELU_N
    sample = "the first 2^22 elements of the batch, repeated"

    def inputs(self):
        rng = np.random.default_rng(0 + self.dist.rank)
        self.host = [rng.uniform(-4, 4, GELU_N).astype(np.float32) for _ in range(3)]

    def config(self):
        return {"workload": self.name, "elements": GELU_N, "seed": 0,
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

    def cpu_step(self, threads: int, oracle) -> float:
        n = 1 << 22
        self.cpu_out = oracle.gelu_chain(self.host[0][:n], self.host[1][:n], self.host[2][:n],
                                         threads=threads)
        return 16.0 * n

    def compare(self) -> float:
        """Max scaled error of the device output against the oracle's on the CPU sample."""
        got = self.out[: self.cpu_out.size].cpu().numpy()
        return float(np.max(np.abs(got - self.cpu_out) / np.maximum(np.abs(self.cpu_out), 1.0)))


class Rows(Workload):
    name = "softmax_layernorm_rows_f32"
    metric = "fused-group GB/s: row softmax -> layernorm, fp32 [65536, 1024]"
    unit = "GB/s"
    dtype = "f32"
    kernel = "softmax_layernorm_k0"
    bytes_per_step = 2 * 4 * ROWS * COLS + 2 * 4 * COLS
    sample = "the first 4096 rows of the batch, repeated"

    def inputs(self):
        rng = np.random.default_rng(0 + self.dist.rank)
        self.x = rng.standard_normal((ROWS, COLS), dtype=np.float32)
        self.gamma = (1 + 0.02 * rng.standard_normal(COLS)).astype(np.float32)
        self.beta = (0.02 * rng.standard_normal(COLS)).astype(np.float32)

    def config(self):
        return {"workload": self.name, "rows": ROWS, "cols": COLS, "seed": 0,
                "bytes_per_step": self.bytes_per_step,
                "l2": "inputs larger than L2 (268 MB read per step), no flush"}

    def setup_device(self, runtime, torch):
        self.module = runtime.load(PREBUILT / "rows" / "rows.json")
        self.dx = torch.from_numpy(self.x).cuda()
        self.dg = torch.from_numpy(self.gamma).cuda()
        self.db = torch.from_numpy(self.beta).cuda()
        self.out = torch.empty_like(self.dx)
        self.px = torch.from_numpy(self.x).pin_memory()
        self.pg = torch.from_numpy(self.gamma).pin_memory()
        self.pb = torch.from_numpy(self.beta).pin_memory()
        self.pout = torch.empty_like(self.px).pin_memory()

    def step_device(self):
        return self.module.device.softmax_layernorm(self.dx, self.dg, self.db, self.out).status

    def step_host(self):
        return self.module.softmax_layernorm(self.px.view(-1), self.pg, self.pb,
                                             self.pout.view(-1)).status

    def h2d_d2h(self):
        return 4 * ROWS * COLS + 8 * COLS, 4 * ROWS * COLS

    def cpu_step(self, threads: int, oracle) -> float:
        rows = 4096
        self.cpu_out = oracle.softmax_layernorm(self.x[:rows], self.gamma, self.beta,
                                                threads=threads)
        return 2.0 * 4 * rows * COLS

    def compare(self) -> float:
        got = self.out[: self.cpu_out.shape[0]].cpu().numpy()
        return float(np.max(np.abs(got - self.cpu_out) / np.maximum(np.abs(self.cpu_out), 1.0)))


class Collatz(Workload):
    name = "collatz_parallel_range"
    metric = "Collatz steps/s: parallel.range(1, 2^26) int64 sum and max of step counts"
    unit = "steps/s"
    dtype = "int64"
    kernel = "par_collatz_collatz_sum_0_part"
    scaling = "strong"
    sample = "the starts [lo, lo + 2^22) of the range, repeated"

    def inputs(self):
        self.lo, self.hi = shard_range(1, COLLATZ_HI, self.dist.world, self.dist.rank)
        self.sum = None

    def config(self):
        return {"workload": self.name, "range": [1, COLLATZ_HI],
                "rank_range": [self.lo, self.hi], "l2": "no data: integer-issue bound"}

    def setup_device(self, runtime, torch):
        self.module = runtime.load(PREBUILT / "collatz" / "collatz.json")
        self.module_lib = runtime.library()

    def step_device(self):
        status, self.sum = self.module.device.collatz_collatz_sum(self.lo, self.hi)
        status2, self.best = self.module.device.collatz_collatz_max(self.lo, self.hi)
        return status or status2

    step_host = step_device

    def units(self) -> float:
        return float(self.sum)

    def job_units(self) -> float:
        return float(self.dist.sum_i64([int(self.sum)])[0])

    def h2d_d2h(self):
        return 32, 16  # (lo, hi) twice in, (sum, max) out

    def roofline(self, kernel_ms: float, peaks: dict) -> dict:
        """Against the step body's issue ceiling, measured here: ppyb200_collatz_step_peak
        runs the same checked-int64 step on four independent chains per lane of a full grid,
        with no divergence (best of 3 launches of 2^12 steps a chain, CUDA events)."""
        import ctypes

        import torch

        lib = self.module_lib
        lib.ppyb200_collatz_step_peak.argtypes = [ctypes.c_int64, ctypes.c_void_p,
                                                  ctypes.c_void_p]
        lib.ppyb200_collatz_step_peak.restype = ctypes.c_int32
        checksum = torch.zeros(1, dtype=torch.int64, device="cuda")
        total = ctypes.c_int64(0)
        best = float("inf")
        for _ in range(4):
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            assert lib.ppyb200_collatz_step_peak(1 << 12, checksum.data_ptr(),
                                                 ctypes.byref(total)) == 0
            e.record()
            torch.cuda.synchronize()
            best = min(best, s.elapsed_time(e))
        peak = total.value / (best / 1e3)
        achieved = self.units() / (kernel_ms / 1e3)
        return {"bound": "int-issue", "achieved": achieved, "peak": peak, "unit": self.unit,
                "frac": achieved / peak, "traffic": None,
                "peak_source": "ppyb200_collatz_step_peak measured in this run: the same "
                               "checked int64 step, 4 chains a lane, no divergence",
                "kernel": self.kernel, "kernel_ms": kernel_ms}

    def cpu_step(self, threads: int, oracle) -> float:
        hi = min(self.hi, self.lo + (1 << 22))
        status, total, best = oracle.collatz(self.lo, hi, threads)
        return float(total)

    def compare(self) -> float:
        return 0.0


class Gemm(Workload):
    name = "matmul_bias_bf16"
    metric = "matmul TFLOP/s: C = A @ B + bias, bf16 A/B, f32 accumulate and C, 8192^3"
    unit = "TFLOP/s"
    dtype = "bf16"
    kernel = "matmul_bf16_pair_kernel"  # K = 8192: CTA pairs
    M = N = K = 8192
    flops = 2 * 8192 ** 3
    sample = "NumPy f32 BLAS on the first 512 rows of A, repeated"

    def inputs(self):
        import torch

        g = torch.Generator().manual_seed(0 + self.dist.rank)
        k = self.K
        self.a = (torch.randn(self.M, k, generator=g) / k ** 0.5).to(torch.bfloat16)
        self.b = (torch.randn(k, self.N, generator=g) / k ** 0.5).to(torch.bfloat16)
        self.bias = 0.02 * torch.randn(self.N, generator=g)

    def config(self):
        return {"workload": self.name, "m": self.M, "n": self.N, "k": self.K,
                "seed": 0, "flops_per_step": self.flops,
                "path": "tensor.matmul of tensor.convert(bf16) + bias through the built module: "
                        "B [K,N] transposed to K-major, then the tcgen05 kernel",
                "l2": "operands 256 MB > L2, no flush"}

    def setup_device(self, runtime, torch):
        import ctypes

        self.module = runtime.load(PREBUILT / "matmul_bf16_8192" / "matmul_bf16_8192.json")
        self.da, self.db, self.dbias = self.a.cuda(), self.b.cuda(), self.bias.cuda()
        self.out = torch.empty(self.M, self.N, device="cuda")
        self.pa, self.pb = self.a.pin_memory(), self.b.pin_memory()
        self.pbias = self.bias.pin_memory()
        self.pout = torch.empty(self.M, self.N).pin_memory()
        self.dbt = self.db.t().contiguous()
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

    def units(self) -> float:
        return float(self.flops)

    def h2d_d2h(self):
        return 2 * 2 * self.M * self.K + 4 * self.N, 4 * self.M * self.N

    def roofline(self, kernel_ms: float, peaks: dict) -> dict:
        achieved = self.flops / (kernel_ms / 1e3) / 1e12
        return {"bound": "tensor", "achieved": achieved, "peak": peaks["bf16_tflops"],
                "unit": "TFLOP/s", "frac": achieved / peaks["bf16_tflops"],
                "traffic": traffic(self.kernel),
                "peak_source": f"{peaks['source']} cuBLAS bf16 (burst)", "kernel": self.kernel,
                "kernel_ms": kernel_ms}

    def cpu_step(self, threads: int, oracle) -> float:
        # NumPy f32 BLAS on the bf16-rounded values (the CPython reference of the path)
        rows = 512
        a = self.a[:rows].float().numpy()
        b = self.b.float().numpy()
        self.cpu_out = a @ b + self.bias.numpy()
        return 2.0 * rows * self.N * self.K

    def compare(self) -> float:
        got = self.out[: self.cpu_out.shape[0]].cpu().numpy().astype(np.float64)
        ref = self.cpu_out.astype(np.float64)
        scale = np.maximum(np.abs(ref), np.sqrt(np.mean(ref ** 2)))
        return float(np.max(np.abs(got - ref) / scale))


class GemmF32(Gemm):
    """The fp32-input variant: C = A @ B + bias with f32 A, B, bias and C at 4096^3, through
    the module the backend builds from tests/golden/matmul_f32_4096.ppyir: a split pass
    (A, B into tf32 high and low parts) and the tcgen05 GEMM over the three products."""

    name = "matmul_bias_f32"
    metric = "matmul TFLOP/s: C = A @ B + bias, f32 A/B/bias/C, 4096^3"
    dtype = "f32"
    kernel = "matmul_tf32x3_pair_kernel"
    M = N = K = 4096
    flops = 2 * 4096 ** 3
    sample = "NumPy f32 BLAS on the first 512 rows of A, repeated"

    def inputs(self):
        import torch

        g = torch.Generator().manual_seed(0 + self.dist.rank)
        k = self.K
        self.a = torch.randn(self.M, k, generator=g) / k ** 0.5
        self.b = torch.randn(k, self.N, generator=g) / k ** 0.5
        self.bias = 0.02 * torch.randn(self.N, generator=g)

    def config(self):
        return {"workload": self.name, "m": self.M, "n": self.N, "k": self.K, "seed": 0,
                "flops_per_step": self.flops,
                "path": "tensor.matmul of f32 operands + bias through the built module: A and B "
                        "split into tf32 high and low parts, then one tcgen05 GEMM over "
                        "A_hi.B_hi + A_hi.B_lo + A_lo.B_hi (K' = 3 K)",
                "l2": "operands 128 MB + split operands 256 MB > L2, no flush"}

    def setup_device(self, runtime, torch):
        self.module = runtime.load(PREBUILT / "matmul_f32_4096" / "matmul_f32_4096.json")
        self.da, self.db, self.dbias = self.a.cuda(), self.b.cuda(), self.bias.cuda()
        self.out = torch.empty(self.M, self.N, device="cuda")
        self.pa, self.pb = self.a.pin_memory(), self.b.pin_memory()
        self.pbias = self.bias.pin_memory()
        self.pout = torch.empty(self.M, self.N).pin_memory()
        self.torch = torch

    kernel_step = None  # the step (split + GEMM + the non-finite check) is the timed launch

    def step_device(self):
        return self.module.device.matmul_bias(self.da, self.db, self.dbias, self.out).status

    def step_host(self):
        return self.module.matmul_bias(self.pa, self.pb, self.pbias, self.pout).status

    def h2d_d2h(self):
        return 2 * 4 * self.M * self.K + 4 * self.N, 4 * self.M * self.N

    def roofline(self, kernel_ms: float, peaks: dict) -> dict:
        # the method's ceiling: three tf32 products at the device's tf32 rate, measured here
        # with cuBLAS (torch.matmul with TF32 allowed, 8192^3, best of 5)
        torch = self.torch
        torch.backends.cuda.matmul.allow_tf32 = True
        x = torch.randn(8192, 8192, device="cuda")
        y = torch.randn(8192, 8192, device="cuda")
        best = float("inf")
        for _ in range(6):
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            torch.matmul(x, y)
            e.record()
            torch.cuda.synchronize()
            best = min(best, s.elapsed_time(e))
        torch.backends.cuda.matmul.allow_tf32 = False
        tf32 = 2 * 8192 ** 3 / (best / 1e3) / 1e12
        achieved = self.flops / (kernel_ms / 1e3) / 1e12
        peak = tf32 / 3
        return {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                "frac": achieved / peak, "traffic": traffic(self.kernel),
                "peak_source": f"cuBLAS tf32 measured in this run ({tf32:.0f} TFLOP/s) / 3 "
                               "products",
                "kernel": "split + " + self.kernel, "kernel_ms": kernel_ms,
                "cublas_tf32_tflops": tf32}


class Gpt2(Workload):
    name = "gpt2_124m_forward"
    metric = "GPT-2-124M forward tokens/s: batch 32 x 1024, f32 logits out"
    unit = "tokens/s"
    dtype = "bf16"
    kernel = "gpt2_forward"
    scaling = "strong"
    BATCH, LENGTH = 32, 1024
    sample = ("torch CPU forward (f32, the reference's ATen ops) of the first sequence "
              "(1 x 1024), repeated")

    def inputs(self):
        import torch

        start, stop = shard_batch(self.BATCH, self.dist.world, self.dist.rank)
        g = torch.Generator().manual_seed(0)
        ids = torch.randint(0, VOCAB, (self.BATCH, self.LENGTH), generator=g)
        self.all_ids = ids
        self.ids = ids[start:stop].contiguous()

    def config(self):
        b = self.ids.shape[0]
        return {"workload": self.name, "batch": self.BATCH, "seq_len": self.LENGTH,
                "layers": 12, "width": 768, "heads": 12, "vocab": VOCAB,
                "parallelism": f"dp{self.dist.world}", "sequences_per_gpu": b,
                "weights": "N(0, 0.02) seed 0, bf16; layernorm, softmax, residual and logits f32",
                "launch": "eager" if self.eager else "one CUDA graph replay per forward",
                "e2e_output": f"all logits: f32 [{b}, {self.LENGTH}, {VOCAB}] per GPU, copied "
                              "into a contiguous pinned host array",
                "l2": "weights 250 MB + activations and 6.6 GB of logits > L2, no flush"}

    def setup_device(self, runtime, torch):
        from ppy_b200 import gpt2

        self.gpt2 = gpt2
        self.torch = torch
        self.model = gpt2.GPT2(gpt2.GPT2_124M, seed=0)
        b = self.ids.shape[0]
        self.stream = torch.cuda.current_stream()
        if self.eager:
            self.dids = self.ids.cuda()
            self.logits = self.model.new_logits(b, self.LENGTH)  # rows on 128-byte lines
            self.slots = [(self.dids, self.logits, None)]
        else:
            # two captured forwards over their own ids and logits buffers (the activations
            # are shared: the replays run one after another on the stream), so that one
            # step's logits can go out over PCIe while the next step computes
            self.slots = []
            for _ in range(2):
                graphed = self.model.graphed(b, self.LENGTH, self.stream)
                graphed.ids.copy_(self.ids)
                self.slots.append((graphed.ids, graphed.logits, graphed))
            self.dids, self.logits, self.graphed = self.slots[0]
        self.pids = self.ids.pin_memory()
        self.host_logits = [torch.empty(b, self.LENGTH, VOCAB).pin_memory()
                            for _ in self.slots]
        self.copy_stream = torch.cuda.Stream()
        self.computed = [torch.cuda.Event() for _ in self.slots]
        self.copied = [torch.cuda.Event() for _ in self.slots]
        self.turn = 0
        self.runtime = runtime

    def _forward(self, slot=0):
        ids, logits, graphed = self.slots[slot]
        if graphed is None:
            self.model.forward(ids, logits)
        else:
            graphed.run()

    def step_device(self):
        self._forward()
        return 0

    def step_host(self):
        """e2e: the step's ids from pinned host memory in, every logit out into a contiguous
        pinned host array. Steps alternate between the two buffer sets; the logits of a step
        go out on a copy stream while the next step computes, and a buffer set is reused
        only after its previous copy-out finished."""
        torch = self.torch
        slot = self.turn % len(self.slots)
        self.turn += 1
        ids, logits, _ = self.slots[slot]
        self.stream.wait_event(self.copied[slot])  # this set's last copy-out is done
        ids.copy_(self.pids, non_blocking=True)
        self._forward(slot)
        self.computed[slot].record(self.stream)
        with torch.cuda.stream(self.copy_stream):
            self.copy_stream.wait_event(self.computed[slot])
            self.runtime.set_stream(self.copy_stream)
            self.runtime.copy_rows_to_host(self.host_logits[slot], logits)
            self.runtime.set_stream(self.stream)
            self.copied[slot].record(self.copy_stream)
        return 0

    def drain(self):
        """The end of the timed host-memory steps waits for the last copy-outs."""
        for event in self.copied:
            self.stream.wait_event(event)

    def finish(self) -> int:
        return self.model.status()

    def units(self) -> float:
        return float(self.ids.numel())

    def job_units(self) -> float:
        return float(self.dist.sum_i64([int(self.units())])[0])

    def h2d_d2h(self):
        b = self.ids.shape[0]
        return 8 * b * self.LENGTH, 4 * b * self.LENGTH * VOCAB

    def roofline(self, kernel_ms: float, peaks: dict) -> dict:
        # per-kernel times from one eager forward with events around every call
        table = self.model.profile(self.dids, self.logits)
        name, (count, ms, flops) = max(table.items(), key=lambda kv: kv[1][1])
        achieved = flops / (ms / 1e3) / 1e12
        peak = peaks["bf16_tflops_sustained"]
        forward_tflops = self.gpt2.sequence_flops(self.gpt2.GPT2_124M, self.ids.shape[0],
                                                  self.LENGTH) / (kernel_ms / 1e3) / 1e12
        line = {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                "frac": achieved / peak, "traffic": traffic(name),
                "peak_source": f"{peaks['source']} cuBLAS bf16 (sustained)", "kernel": name,
                "kernel_ms": ms / count, "forward_ms": kernel_ms,
                "forward_tflops": forward_tflops, "forward_frac": forward_tflops / peak,
                "breakdown_ms": {k: round(v[1], 3) for k, v in table.items()}}
        if self.dist.world == 1:
            line["like_for_like"] = torch_bf16_forward_ms(self.model, self.dids)
        return line

    def cpu_step(self, threads: int, oracle) -> float:
        import torch

        from oracle import gpt2 as oracle_gpt2

        if not hasattr(self, "cpu_model"):
            self.cpu_model = oracle_gpt2.cpu_model(seed=0)
        torch.set_num_threads(threads)
        with torch.no_grad():
            self.cpu_out = self.cpu_model(self.all_ids[:1])
        return float(self.LENGTH)

    def compare(self) -> float:
        """Max error of sequence 0's logits, as the last host-memory step copied them out,
        against the CPU forward, per element against max(|ref|, rms of ref)."""
        self.torch.cuda.synchronize()
        slot = (self.turn - 1) % len(self.slots)
        got = self.host_logits[slot][0].double()
        ref = self.cpu_out[0].double()
        scale = torch_max(ref.abs(), ref.pow(2).mean().sqrt())
        return float(((got - ref).abs() / scale).max())


def torch_bf16_forward_ms(model, ids, steps: int = 5) -> dict:
    """The same GPT-2 forward written with torch's own bf16 operators -- cuBLAS GEMMs through
    F.linear, F.scaled_dot_product_attention (its fused flash kernel), F.layer_norm and
    F.gelu -- on the same weights and ids: the like-for-like comparison a torch user would
    run. Eager, and replayed from a CUDA graph; bf16 logits (what torch gives for bf16
    operands). A measurement beside the product path, not part of it."""
    import torch
    import torch.nn.functional as F

    cfg = model.config
    c, heads, hd = cfg.width, cfg.heads, cfg.head_dim
    blocks = [{k: (v.to(torch.bfloat16) if v.dtype != torch.bfloat16 else v)
               for k, v in blk.items()} for blk in model.blocks]
    lnf_g, lnf_b = model.lnf_g.to(torch.bfloat16), model.lnf_b.to(torch.bfloat16)

    def forward(tokens):
        b, n = tokens.shape
        x = model.wte[tokens] + model.wpe[:n]
        for blk in blocks:
            h = F.layer_norm(x, (c,), blk["ln1_g"], blk["ln1_b"], 1e-5)
            q, k, v = F.linear(h, blk["w_qkv"], blk["b_qkv"]).split(c, dim=-1)
            shape = lambda t: t.view(b, n, heads, hd).transpose(1, 2)  # noqa: E731
            a = F.scaled_dot_product_attention(shape(q), shape(k), shape(v), is_causal=True)
            x = x + F.linear(a.transpose(1, 2).reshape(b, n, c), blk["w_o"], blk["b_o"])
            h = F.layer_norm(x, (c,), blk["ln2_g"], blk["ln2_b"], 1e-5)
            f = F.gelu(F.linear(h, blk["w_fc"], blk["b_fc"]), approximate="tanh")
            x = x + F.linear(f, blk["w_proj"], blk["b_proj"])
        return F.layer_norm(x, (c,), lnf_g, lnf_b, 1e-5) @ model.wte.t()

    def timed(fn) -> float:
        for _ in range(2):
            fn()
        torch.cuda.synchronize()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(steps):
            fn()
        end.record()
        torch.cuda.synchronize()
        return start.elapsed_time(end) / steps

    with torch.no_grad():
        eager = timed(lambda: forward(ids))
        graph = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            forward(ids)
        torch.cuda.current_stream().wait_stream(side)
        with torch.cuda.graph(graph):
            out = forward(ids)
        replayed = timed(graph.replay)
        del out, graph
    torch.cuda.empty_cache()
    tokens = ids.numel()
    return {"torch_bf16_eager_ms": eager, "torch_bf16_graph_ms": replayed,
            "torch_bf16_graph_tokens_per_s": tokens / (replayed / 1e3),
            "what": "the same forward with torch's bf16 operators (cuBLAS F.linear, SDPA flash "
                    "attention, layer_norm, gelu), bf16 logits, same weights and ids, on this "
                    "GPU"}


def torch_max(a, b):
    import torch

    return torch.maximum(a, b)


class Gpt2TP(Gpt2):
    """The tensor-parallel variant: the ranks of a group work on the group's sequences with
    12/T heads, 3072/T hidden units and 50257/T logits columns each, two all-reduces of the
    residual stream per block (T in {1, 2, 4}); N ranks form N/T such groups, each with its
    share of the batch (8 GPUs: 2 groups of 4). `--tp` picks T, 0 the widest that fits."""

    name = "gpt2_124m_forward_tp"
    metric = "GPT-2-124M forward tokens/s, tensor parallel: batch 32 x 1024, f32 logits out"
    kernel = "gpt2_tp_forward"

    def inputs(self):
        import torch

        from ppy_b200 import gpt2, gpt2_tp

        self.dp, self.tp = gpt2_tp.hybrid_layout(self.dist.world, gpt2.GPT2_124M, self.tp)
        start, stop = shard_batch(self.BATCH, self.dp, self.dist.rank // self.tp)
        g = torch.Generator().manual_seed(0)
        ids = torch.randint(0, VOCAB, (self.BATCH, self.LENGTH), generator=g)
        self.all_ids = ids
        self.ids = ids[start:stop].contiguous()

    def config(self):
        cfg = super().config()
        tokens = self.ids.numel()
        if self.exchange == "nvlink":
            exchange = (f"fused reduce-scatter + all-gather over NVLink in each group of "
                        f"{self.tp}: each row-parallel GEMM's epilogue stores the rows of the "
                        f"f32 [{tokens}, 768] partial owned by rank s into rank s's buffer, a "
                        "flag per rank, the owner's in-order sum of its block sent to every "
                        "rank, a second flag round; 2 per block")
        else:
            exchange = (f"2 NCCL all-reduces (sum, f32 [{tokens}, 768]) per block inside "
                        f"each group of {self.tp}")
        cfg.update(workload=self.name,
                   parallelism=f"tp{self.tp}" if self.dp == 1 else f"dp{self.dp}xtp{self.tp}",
                   exchange=exchange, launch="eager",
                   e2e_output="this rank's logits columns, copied into a contiguous pinned host "
                              "array")
        return cfg

    def setup_device(self, runtime, torch):
        from ppy_b200 import gpt2, gpt2_tp

        group = None
        if self.dist.world > 1:
            group, _ = gpt2_tp.hybrid_groups(self.tp)
        self.model = gpt2_tp.GPT2TensorParallel(gpt2.GPT2_124M, seed=0, group=group,
                                                exchange=self.exchange)
        self.gpt2 = gpt2
        self.torch = torch
        self.eager = True
        self.stream = torch.cuda.current_stream()
        self.dids = self.ids.cuda()
        self.pids = self.ids.pin_memory()
        v0, v1 = self.model.shard.vocab
        b = self.ids.shape[0]
        self.logits = self.model.new_logits(b, self.LENGTH)  # rows on 128-byte lines
        self.slots = [(self.dids, self.logits, None)]
        self.host_logits = [torch.empty(b, self.LENGTH, v1 - v0).pin_memory()]
        self.copy_stream = torch.cuda.Stream()
        self.computed = [torch.cuda.Event()]
        self.copied = [torch.cuda.Event()]
        self.turn = 0
        self.runtime = runtime

    def _forward(self, slot=0):
        self.model.forward(self.dids, self.logits)

    def job_units(self) -> float:
        return float(self.units()) * self.dp  # the ranks of a group share their tokens

    def h2d_d2h(self):
        v0, v1 = self.model.shard.vocab
        b = self.ids.shape[0]
        return 8 * b * self.LENGTH, 4 * b * self.LENGTH * (v1 - v0)

    def roofline(self, kernel_ms: float, peaks: dict) -> dict:
        peak = peaks["bf16_tflops_sustained"]
        per_gpu = self.gpt2.sequence_flops(self.gpt2.GPT2_124M, self.BATCH, self.LENGTH) / (
            self.dist.world) / (kernel_ms / 1e3) / 1e12
        return {"bound": "tensor", "achieved": per_gpu, "peak": peak, "unit": "TFLOP/s",
                "frac": per_gpu / peak, "traffic": None,
                "peak_source": f"{peaks['source']} cuBLAS bf16 (sustained)",
                "kernel": self.kernel, "kernel_ms": kernel_ms}

    def compare(self) -> float:
        v0, v1 = self.model.shard.vocab
        self.torch.cuda.synchronize()
        got = self.host_logits[0][0].double()
        ref = self.cpu_out[0, :, v0:v1].double()
        scale = torch_max(ref.abs(), ref.pow(2).mean().sqrt())
        return float(((got - ref).abs() / scale).max())


WORKLOADS = {"gpt2": Gpt2, "gpt2_tp": Gpt2TP, "gelu": Gelu, "rows": Rows, "collatz": Collatz,
             "gemm": Gemm, "gemm_f32": GemmF32}


def to_metric(w: Workload, units: float, seconds: float) -> float:
    if w.unit == "GB/s":
        return units / seconds / 1e9
    if w.unit == "TFLOP/s":
        return units / seconds / 1e12
    return units / seconds


def cpu_baseline(w: Workload, seconds: float) -> dict:
    """The oracle (or, for GPT-2, the reference's torch path) on the host cores over a
    bounded sample, and the device output's error against it on that sample."""
    import oracle

    threads = oracle.threads_available()
    done = 0.0
    steps = 0
    start = time.perf_counter()
    while True:
        done += w.cpu_step(threads, oracle)
        steps += 1
        elapsed = time.perf_counter() - start
        if elapsed >= seconds:
            break
    return {"value": to_metric(w, done, elapsed), "unit": w.unit, "cores": threads,
            "kind": "port", "sample": f"{w.sample}; {steps} passes in {elapsed:.1f} s",
            "max_rel_error_vs_device": w.compare()}


# ---------------------------------------------------------------- the reference arm


def run_reference(args, dist: Dist) -> None:
    dist.start("gloo")
    if dist.rank != 0:
        dist.stop()
        return
    import oracle

    threads = oracle.threads_available()

    def time_cpu(name: str, steps: int, warmup: int) -> tuple[Workload, float, float]:
        w = WORKLOADS[name](dist)
        w.dist.world = 1
        w.inputs()
        for _ in range(warmup):
            w.cpu_step(threads, oracle)
        units = 0.0
        start = time.perf_counter()
        for _ in range(steps):
            units += w.cpu_step(threads, oracle)
        elapsed = time.perf_counter() - start
        return w, to_metric(w, units, elapsed), elapsed

    w, value, elapsed = time_cpu(args.workload, args.steps, args.warmup)
    line = {"metric": w.metric, "value": value, "unit": w.unit, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": elapsed / max(args.steps, 1) * 1e3, "higher_is_better": True,
            "scaling": w.scaling, "vs_baseline": None, "dtype": w.dtype, "data": "synthetic",
            "config": w.config(), "impl": "reference",
            "cpu_baseline": {"value": value, "unit": w.unit, "cores": threads, "kind": "port",
                             "sample": f"one bounded sample per step: {w.sample}"},
            "e2e": {"value": value, "unit": w.unit, "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    extras = _extras(args)
    if extras:
        line["workloads"] = {}
        for name in extras:
            x, xv, _ = time_cpu(name, 10, 1)
            line["workloads"][x.name] = {"metric": x.metric, "value": xv, "unit": x.unit,
                                         "impl": "reference", "cores": threads,
                                         "kind": "port", "sample": x.sample}
    print(json.dumps(line), flush=True)
    dist.stop()


# ---------------------------------------------------------------- the B200 arm


def _extras(args) -> list[str]:
    if args.workload != "gpt2" or args.extras in ("", "none"):
        return []
    return [x for x in args.extras.split(",") if x]


def measure(w: Workload, steps: int, warmup: int, dist: Dist, stream, runtime, torch,
            clocks: Clocks, peaks: dict) -> dict:
    """Warm up, then time `steps` device-resident steps and `steps` host-memory steps, each
    between one pair of CUDA events on `stream`, bracketed by a barrier and a synchronize;
    the time is the max over ranks. Returns the workload's figures."""
    for _ in range(max(warmup, 3)):
        assert w.step_device() == 0
        assert w.step_host() == 0
    torch.cuda.synchronize()
    launches0 = runtime.launches()

    def timed(step) -> float:
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        dist.barrier()
        torch.cuda.synchronize()
        begin = time.perf_counter()
        start.record(stream)
        for _ in range(steps):
            if step() != 0:
                raise SystemExit(f"{w.name}: a step failed")
        if getattr(w, "drain", None) is not None:
            w.drain()  # work the steps left on other streams ends inside the timed region
        end.record(stream)
        torch.cuda.synchronize()
        dist.barrier()
        clocks.mark(begin, time.perf_counter())
        return dist.max(start.elapsed_time(end))

    device_ms = timed(w.step_device)
    if getattr(w, "finish", None) is not None and w.finish() != 0:
        raise SystemExit(f"{w.name}: a kernel raised its status word")
    # the dominant kernel's own launch duration, for workloads whose step is more than it
    kernel_ms = device_ms / steps
    if getattr(w, "kernel_step", None) is not None:
        k0 = torch.cuda.Event(enable_timing=True)
        k1 = torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        k0.record(stream)
        for _ in range(steps):
            if w.kernel_step() != 0:
                raise SystemExit(f"{w.name}: the kernel step failed")
        k1.record(stream)
        torch.cuda.synchronize()
        kernel_ms = k0.elapsed_time(k1) / steps
    e2e_ms = timed(w.step_host)
    launches = runtime.launches() - launches0
    job = w.job_units()
    h2d, d2h = w.h2d_d2h()
    result = {"metric": w.metric, "value": to_metric(w, job * steps, device_ms / 1e3),
              "unit": w.unit, "ms_per_step": device_ms / steps, "steps": steps,
              "scaling": w.scaling, "dtype": w.dtype, "config": w.config(),
              "e2e": {"value": to_metric(w, job * steps, e2e_ms / 1e3), "unit": w.unit,
                      "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                      "ms_per_step": e2e_ms / steps},
              "gpu_launches": int(launches)}
    if dist.rank == 0:
        result["roofline"] = w.roofline(kernel_ms, peaks)
    return result


def run_b200(args, dist: Dist) -> None:
    import torch

    from ppy_b200 import runtime

    torch.cuda.set_device(dist.local)
    dist.start("nccl")
    runtime.init(dist.local)
    # one stream for everything: the launches, copies, graph replays and the timing events
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    runtime.set_stream(stream)
    peaks = measured_peaks()
    clocks = Clocks(dist.local)
    clocks.start()

    def make(name: str) -> Workload:
        w = WORKLOADS[name](dist)
        w.tp, w.exchange, w.eager = args.tp, args.exchange, args.eager
        w.inputs()
        w.setup_device(runtime, torch)
        return w

    main = make(args.workload)
    result = measure(main, args.steps, args.warmup, dist, stream, runtime, torch, clocks, peaks)
    main_windows = list(clocks.windows)
    extras = []
    for name in _extras(args):
        x = make(name)
        extras.append((x, measure(x, max(args.steps, 100), args.warmup, dist, stream, runtime,
                                  torch, clocks, peaks)))
    clocks.stop()
    if dist.rank == 0:
        line = {"metric": main.metric, "value": result["value"], "unit": main.unit,
                "n_gpus": dist.world, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": result["ms_per_step"], "higher_is_better": True,
                "scaling": main.scaling, "vs_baseline": None, "dtype": main.dtype,
                "data": "synthetic (seeded)", "config": main.config(), "e2e": result["e2e"],
                "gpu_launches": result["gpu_launches"] + sum(r["gpu_launches"] for _, r in extras),
                "clocks": clocks.summary(main_windows), "roofline": result["roofline"]}
        if dist.world == 1:
            line["cpu_baseline"] = cpu_baseline(main, args.cpu_seconds)
        if extras:
            line["workloads"] = {}
            for x, r in extras:
                entry = dict(r)
                if dist.world == 1:
                    entry["cpu_baseline"] = cpu_baseline(x, args.cpu_seconds)
                line["workloads"][x.name] = entry
            line["workloads_clocks"] = clocks.summary(clocks.windows[len(main_windows):])
        print(json.dumps(line), flush=True)
    close = getattr(getattr(main, "model", None), "close", None)
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
