"""GPT-2 forward on the b200 kernels (the model of examples/46_gpt2/gpt2.ppy in the reference).

torch is storage only: weights and activations are torch CUDA tensors, and every operation
of the forward is one of this package's kernels, called through the C ABI:

    embed (gather)                         ppyb200_gpt2_embed
    per block: layernorm -> bf16           the row kernel the backend builds from
                                           tests/golden/gpt2_layernorm.ppyir
               QKV = h Wqkv^T + b          ppyb200_linear_qkv_bf16 (tcgen05; q, k as is,
                                           v transposed per head)
               causal attention            ppyb200_attention_causal_vt_bf16 (tcgen05)
               x += a Wo^T + b             ppyb200_linear_residual (tcgen05, residual in place)
               layernorm -> bf16
               f = gelu(n Wfc^T + b)       ppyb200_linear_bf16 (GELU-tanh epilogue)
               x += f Wproj^T + b          ppyb200_linear_residual
    final layernorm, logits = n wte^T      ppyb200_matmul_bf16_kmajor (tied head, N = 50257)

Weights are bf16 in torch.nn.Linear's [out, in] layout (K-major for the tensor cores); the
residual stream, layernorm and softmax arithmetic and the logits are f32. The q, k, v
projections of the reference (three [width, width] weights) are one [3 width, width] weight
here, the same numbers side by side.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass
from pathlib import Path

from . import runtime

__all__ = ["Config", "GPT2", "GPT2_124M", "GraphedForward"]

PREBUILT = Path(__file__).resolve().parent / "prebuilt"


@dataclass(frozen=True)
class Config:
    layers: int = 12
    width: int = 768
    heads: int = 12
    vocab: int = 50257
    context: int = 1024

    @property
    def head_dim(self) -> int:
        return self.width // self.heads


GPT2_124M = Config()


def _bind(lib) -> None:
    if getattr(lib, "_gpt2_bound", False):
        return
    p, i64, i32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32
    lib.ppyb200_gpt2_embed.argtypes = [p, p, p, p, i64, i64, i64, i64, p]
    lib.ppyb200_linear_bf16.argtypes = [p, p, p, p, i64, i64, i64, i32, p]
    lib.ppyb200_linear_residual.argtypes = [p, p, p, p, i64, i64, i64, p]
    lib.ppyb200_linear_qkv_bf16.argtypes = [p, p, p, p, p, i64, i64, i64, i64, p]
    lib.ppyb200_attention_causal_bf16.argtypes = [p, p, i64, i64, i64, i64]
    lib.ppyb200_attention_causal_vt_bf16.argtypes = [p, p, p, i64, i64, i64, i64, p]
    lib.ppyb200_matmul_bf16_kmajor.argtypes = [p, p, p, p, i64, i64, i64]
    lib.ppyb200_matmul_bf16_kmajor_ld.argtypes = [p, p, p, p, i64, i64, i64, i64]
    for name in ("ppyb200_gpt2_embed", "ppyb200_linear_bf16", "ppyb200_linear_residual",
                 "ppyb200_linear_qkv_bf16", "ppyb200_attention_causal_bf16",
                 "ppyb200_attention_causal_vt_bf16", "ppyb200_matmul_bf16_kmajor",
                 "ppyb200_matmul_bf16_kmajor_ld"):
        getattr(lib, name).restype = i32
    lib._gpt2_bound = True


class GPT2:
    """A randomly initialised GPT-2 (N(0, 0.02) weights from `seed`, zero biases, unit
    layernorm gains), resident on the current CUDA device."""

    def __init__(self, config: Config = GPT2_124M, seed: int = 0, device: str = "cuda") -> None:
        import torch

        self.config = config
        self.device = device
        c, v = config.width, config.vocab
        g = torch.Generator().manual_seed(seed)

        def normal(*shape):
            return (0.02 * torch.randn(*shape, generator=g)).to(torch.bfloat16).to(device)

        def zeros(n):
            return torch.zeros(n, dtype=torch.float32, device=device)

        def ones(n):
            return torch.ones(n, dtype=torch.float32, device=device)

        self.wte = normal(v, c)
        self.wpe = normal(config.context, c)
        self.blocks = []
        for _ in range(config.layers):
            self.blocks.append({
                "ln1_g": ones(c), "ln1_b": zeros(c),
                "w_qkv": normal(3 * c, c), "b_qkv": zeros(3 * c),
                "w_o": normal(c, c), "b_o": zeros(c),
                "ln2_g": ones(c), "ln2_b": zeros(c),
                "w_fc": normal(4 * c, c), "b_fc": zeros(4 * c),
                "w_proj": normal(c, 4 * c), "b_proj": zeros(c),
            })
        self.lnf_g, self.lnf_b = ones(c), zeros(c)
        self.lib = runtime.library()
        _bind(self.lib)
        self.layernorm = runtime.load(PREBUILT / "gpt2_layernorm" / "gpt2_layernorm.json")
        self._buffers: dict = {}

    def _scratch(self, tokens: int):
        import torch

        found = self._buffers.get(tokens)
        if found is None:
            c, v, d = self.config.width, self.config.vocab, self.device
            found = {
                "x": torch.empty(tokens, c, dtype=torch.float32, device=d),
                "h": torch.empty(tokens, c, dtype=torch.bfloat16, device=d),
                "qkv": torch.empty(tokens, 3 * c, dtype=torch.bfloat16, device=d),
                "vt": torch.empty(tokens * c, dtype=torch.bfloat16, device=d),
                "att": torch.empty(tokens, c, dtype=torch.bfloat16, device=d),
                "f": torch.empty(tokens, 4 * c, dtype=torch.bfloat16, device=d),
                "status": torch.zeros(1, dtype=torch.int32, device=d),
            }
            self._buffers = {tokens: found}
        return found

    def _check(self, status: int, what: str) -> None:
        if status != runtime.STATUS_OK:
            raise runtime.B200Error(f"{what}: {runtime.last_error()}")

    def new_logits(self, batch: int, length: int):
        """An f32 [batch, length, vocab] tensor whose rows start on 128-byte lines: a view of
        [batch, length, vocab rounded up to 32] (50272 for 50257), so that the LM head stores
        whole lines (a 50257-float row starts anywhere in a line and splits every store over
        two). Values live in the first `vocab` columns only."""
        import torch

        v = self.config.vocab
        pitch = (v + 31) // 32 * 32
        rows = torch.empty(batch, length, pitch, dtype=torch.float32, device=self.device)
        return rows[:, :, :v]

    @staticmethod
    def _row_pitch(logits, batch: int, length: int, vocab: int, device: str = "cuda") -> int:
        """The distance between consecutive logits rows, in floats, of a [batch, length, vocab]
        f32 tensor on `device` whose rows are evenly spaced (contiguous, or a view such as
        new_logits)."""
        import torch

        if (tuple(logits.shape) != (batch, length, vocab) or logits.dtype != torch.float32
                or logits.device.type != device or logits.stride(2) != 1):
            raise runtime.B200Error(f"logits: f32 [{batch}, {length}, {vocab}] on {device}, "
                                    "unit stride along the vocabulary")
        pitch = logits.stride(1)
        if pitch < vocab or (batch > 1 and logits.stride(0) != length * pitch):
            raise runtime.B200Error("logits: rows evenly spaced, at least vocab floats apart")
        return pitch

    def forward(self, ids, logits=None):
        """Logits [batch, length, vocab] (f32) for token ids [batch, length] (int64, CUDA),
        into `logits` when given (any evenly spaced rows), else into new_logits()."""
        cfg = self.config
        batch, length = ids.shape
        tokens = batch * length
        c, v = cfg.width, cfg.vocab
        if length > cfg.context or length % 128 != 0:
            raise runtime.B200Error("the sequence length is a multiple of 128 up to the context")
        ids = ids.contiguous()
        s = self._scratch(tokens)
        x, h, qkv, vt, att, f = s["x"], s["h"], s["qkv"], s["vt"], s["att"], s["f"]
        status = s["status"]
        if logits is None:
            logits = self.new_logits(batch, length)
        pitch = self._row_pitch(logits, batch, length, v)
        lib = self.lib
        st = status.data_ptr()
        status.zero_()
        self._check(lib.ppyb200_gpt2_embed(ids.data_ptr(), self.wte.data_ptr(),
                                           self.wpe.data_ptr(), x.data_ptr(), tokens, length, c,
                                           v, st), "embed")
        ln = self.layernorm.device.layernorm_bf16
        for blk in self.blocks:
            self._check(ln(x, blk["ln1_g"], blk["ln1_b"], h).status, "layernorm")
            self._check(lib.ppyb200_linear_qkv_bf16(h.data_ptr(), blk["w_qkv"].data_ptr(),
                                                    blk["b_qkv"].data_ptr(), qkv.data_ptr(),
                                                    vt.data_ptr(), tokens, c, length, cfg.heads,
                                                    st), "qkv")
            self._check(lib.ppyb200_attention_causal_vt_bf16(qkv.data_ptr(), vt.data_ptr(),
                                                             att.data_ptr(), batch, length,
                                                             cfg.heads, cfg.head_dim, st),
                        "attention")
            self._check(lib.ppyb200_linear_residual(att.data_ptr(), blk["w_o"].data_ptr(),
                                                    blk["b_o"].data_ptr(), x.data_ptr(), tokens,
                                                    c, c, st), "out projection")
            self._check(ln(x, blk["ln2_g"], blk["ln2_b"], h).status, "layernorm")
            self._check(lib.ppyb200_linear_bf16(h.data_ptr(), blk["w_fc"].data_ptr(),
                                                blk["b_fc"].data_ptr(), f.data_ptr(), tokens,
                                                4 * c, c, 1, st), "fc")
            self._check(lib.ppyb200_linear_residual(f.data_ptr(), blk["w_proj"].data_ptr(),
                                                    blk["b_proj"].data_ptr(), x.data_ptr(),
                                                    tokens, c, 4 * c, st), "proj")
        self._check(ln(x, self.lnf_g, self.lnf_b, h).status, "layernorm")
        self._check(lib.ppyb200_matmul_bf16_kmajor_ld(h.data_ptr(), self.wte.data_ptr(), None,
                                                      logits.data_ptr(), pitch, tokens, v, c),
                    "lm head")
        return logits

    def profile(self, ids, logits=None) -> dict:
        """One forward with CUDA events around every call: {kernel: [launches, ms, flops]}.
        Not for timing the whole forward (the events serialise nothing but add records)."""
        import torch

        cfg = self.config
        batch, length = ids.shape
        tokens, c, v = batch * length, cfg.width, cfg.vocab
        stream = torch.cuda.current_stream()
        table: dict = {}
        marks: list = []
        calls = {"qkv": 2 * tokens * c * 3 * c, "out": 2 * tokens * c * c,
                 "fc": 2 * tokens * c * 4 * c, "proj": 2 * tokens * 4 * c * c,
                 "attention": attention_flops(cfg, batch, length) / cfg.layers,
                 "layernorm": 0, "embed": 0, "lm_head": 2 * tokens * c * v}
        lib = self.lib
        original = {}

        def wrap(name, fn):
            def timed(*args):
                start = torch.cuda.Event(enable_timing=True)
                end = torch.cuda.Event(enable_timing=True)
                start.record(stream)
                result = fn(*args)
                end.record(stream)
                marks.append((name, start, end))
                return result
            return timed

        names = {"ppyb200_gpt2_embed": "embed", "ppyb200_linear_qkv_bf16": "qkv",
                 "ppyb200_attention_causal_vt_bf16": "attention",
                 "ppyb200_matmul_bf16_kmajor_ld": "lm_head"}
        for symbol, name in names.items():
            original[symbol] = getattr(lib, symbol)
        linear = lib.ppyb200_linear_bf16
        residual = lib.ppyb200_linear_residual

        class _Lib:
            pass

        shim = _Lib()
        for symbol, name in names.items():
            setattr(shim, symbol, wrap(name, original[symbol]))
        shim.ppyb200_linear_bf16 = lambda *a: wrap("fc", linear)(*a)
        shim.ppyb200_linear_residual = lambda *a: wrap(
            "proj" if a[6] == 4 * c else "out", residual)(*a)
        ln = self.layernorm
        self.lib = shim
        device_ns = ln.device
        plain = device_ns.layernorm_bf16
        device_ns.layernorm_bf16 = wrap("layernorm", plain)
        try:
            self.forward(ids, logits)
        finally:
            self.lib = lib
            device_ns.layernorm_bf16 = plain
        torch.cuda.synchronize()
        for name, start, end in marks:
            entry = table.setdefault(name, [0, 0.0, 0.0])
            entry[0] += 1
            entry[1] += start.elapsed_time(end)
            entry[2] += calls[name]
        return table

    def status(self) -> int:
        """The device status word of the last forward (0 OK; 2 a kernel raised). Syncs."""
        for buffers in self._buffers.values():
            return int(buffers["status"].item())
        return 0

    def graphed(self, batch: int, length: int, stream) -> "GraphedForward":
        """The forward over fixed device buffers of `batch` x `length` token ids, captured
        once on `stream` into a CUDA graph (see GraphedForward)."""
        return GraphedForward(self, batch, length, stream)


class GraphedForward:
    """One GPT-2 forward captured into a CUDA graph: `ids` (int64 [batch, length]) in,
    `logits` (f32 [batch, length, vocab], rows 128-byte aligned as new_logits) out, both
    fixed device buffers. `run()` replays every kernel of the forward with one host call, so
    the host's launch cost (about 90 C-ABI calls) drops out of the step: with few tokens per
    GPU the kernels are short enough for it to matter. The graph is captured on `stream`
    after one plain forward (which sets up the scratch buffers and each kernel's launch
    attributes); replays go to `stream` too."""

    def __init__(self, model: GPT2, batch: int, length: int, stream) -> None:
        import torch

        self.model = model
        self.stream = stream
        self.ids = torch.zeros(batch, length, dtype=torch.int64, device=model.device)
        self.logits = model.new_logits(batch, length)
        runtime.set_stream(stream)
        with torch.cuda.stream(stream):
            model.forward(self.ids, self.logits)
        stream.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        before = runtime.launches()
        with torch.cuda.graph(self.graph, stream=stream):
            runtime.set_stream(stream)
            model.forward(self.ids, self.logits)
        runtime.set_stream(stream)
        self.launches = runtime.launches() - before  # kernels one replay runs

    def run(self):
        """Replay the forward on the stream; counts its kernels as launched."""
        self.graph.replay()
        runtime.count_launches(self.launches)
        return self.logits

    def status(self) -> int:
        """The device status word of the last replay (0 OK; 2 a kernel raised). Syncs."""
        return self.model.status()


def attention_flops(config: Config, batch: int, length: int) -> float:
    """QK^T and PV FLOPs of causal attention over all layers (the causal half)."""
    return config.layers * batch * config.heads * 2 * 2 * config.head_dim * length * (length + 1) / 2


def sequence_flops(config: Config, batch: int, length: int) -> float:
    """Matmul FLOPs of one forward: block GEMMs, causal attention, the tied LM head."""
    tokens = batch * length
    w = config.width
    gemm = tokens * config.layers * 2 * (3 * w * w + w * w + 8 * w * w)
    head = tokens * 2 * w * config.vocab
    return gemm + head + attention_flops(config, batch, length)

