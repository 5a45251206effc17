"""Tensor-parallel GPT-2 forward over g GPUs (one process per GPU; torch.distributed with NCCL
for the exchange), the TP variant of the reference's GPT-2 example
(examples/46_gpt2/gpt2.ppy:18-57, block; :210-241, forward).

Each rank holds 12/g heads and 3072/g hidden units of every block and 50257/g rows of the tied
LM head:

    QKV projection   column-parallel: this rank's q, k, v heads (ppyb200_linear_qkv_bf16)
    attention        on the local heads (ppyb200_attention_causal_vt_bf16)
    out projection   row-parallel: rank 0 adds its partial product, the bias and the residual
                     into x (ppyb200_linear_residual), the other ranks write their partial
                     product into x (ppyb200_matmul_bf16_kmajor); one all-reduce (sum) of x
    FC + GELU        column-parallel (ppyb200_linear_bf16, GELU epilogue)
    proj             row-parallel, as the out projection; one all-reduce of x
    layernorms       replicated on the full residual stream
    LM head          vocab-parallel: this rank's slice of the logits

Two all-reduces of the f32 residual stream [tokens, 768] per block: NCCL's after each
row-parallel GEMM (`exchange="nccl"`), or, with `exchange="nvlink"`, none at all -- a
reduce-scatter and an all-gather over NVLink peer memory (csrc/tp_exchange.cu): the GEMM's
epilogue stores the tile rows of row block s into rank s's exchange buffer, a flag per rank
marks them complete, rank s adds the bias and the g partials of its block to its residual stream
in rank order and stores the sum into every rank's gather buffer, and a second round of flags
lets each rank copy the other blocks in (the same sum, bit for bit, on every rank). g divides
12 and the local widths (768/g and 3072/g) stay multiples of 64 (the tensor-core K step): g in
{1, 2, 4}. More
ranks than that run as data-parallel groups of tensor-parallel ranks (`hybrid_layout`,
`hybrid_groups`): 8 GPUs as 2 groups of 4, each group with half the batch.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

from . import runtime
from .gpt2 import GPT2, GPT2_124M, Config, _bind

__all__ = ["TPShard", "splits", "shard_ranges", "hybrid_layout", "hybrid_groups", "shard_block",
           "GPT2TensorParallel"]


@dataclass(frozen=True)
class TPShard:
    """The slices rank `rank` of `size` holds."""

    rank: int
    size: int
    heads: tuple[int, int]   # [first, last) head
    hidden: tuple[int, int]  # [first, last) FC unit
    vocab: tuple[int, int]   # [first, last) LM head row


def splits(config: Config, size: int) -> bool:
    """Whether `size` ranks split the heads, and the widths into whole 64-wide K steps."""
    return (size >= 1 and config.heads % size == 0 and config.width % size == 0
            and (config.width // size) % 64 == 0 and (4 * config.width // size) % 64 == 0)


def shard_ranges(config: Config, rank: int, size: int) -> TPShard:
    if size < 1 or not 0 <= rank < size:
        raise ValueError(f"rank {rank} of {size}")
    if not splits(config, size):
        raise ValueError(f"{size} ranks do not split {config.heads} heads and the widths "
                         f"into 64-wide slices")
    hl = config.heads // size
    fl = 4 * config.width // size
    per, extra = divmod(config.vocab, size)
    v0 = rank * per + min(rank, extra)
    return TPShard(rank, size, (rank * hl, (rank + 1) * hl), (rank * fl, (rank + 1) * fl),
                   (v0, v0 + per + (1 if rank < extra else 0)))


def _bind_exchange(lib) -> None:
    if getattr(lib, "_exchange_bound", False):
        return
    p, i64, i32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32
    lib.ppyb200_shared_alloc.argtypes = [i64, p]
    lib.ppyb200_shared_alloc.restype = p
    lib.ppyb200_shared_open.argtypes = [p]
    lib.ppyb200_shared_open.restype = p
    lib.ppyb200_shared_close.argtypes = [p]
    lib.ppyb200_shared_close.restype = None
    lib.ppyb200_shared_free.argtypes = [p]
    lib.ppyb200_shared_free.restype = None
    lib.ppyb200_tp_partial_scatter.argtypes = [p, p, p, i32, i64, i64, i64, p]
    lib.ppyb200_tp_signal.argtypes = [p, i32, i32, i32]
    lib.ppyb200_tp_accumulate.argtypes = [p, p, p, p, i32, i64, i64, i32, p]
    lib.ppyb200_tp_partial_reduce_scatter.argtypes = [p, p, p, i32, i64, i64, i64, p]
    lib.ppyb200_tp_reduce_block.argtypes = [p, p, p, p, p, i32, i32, i64, i64, i32, p]
    lib.ppyb200_tp_gather_blocks.argtypes = [p, p, p, i32, i32, i64, i64, i32, p]
    for name in ("ppyb200_tp_partial_scatter", "ppyb200_tp_signal", "ppyb200_tp_accumulate",
                 "ppyb200_tp_partial_reduce_scatter", "ppyb200_tp_reduce_block",
                 "ppyb200_tp_gather_blocks"):
        getattr(lib, name).restype = i32
    lib._exchange_bound = True


def hybrid_layout(world: int, config: Config = GPT2_124M, tp: int = 0) -> tuple[int, int]:
    """(dp, tp): `world` ranks as dp = world / tp groups of tp consecutive ranks, each group
    tensor-parallel over its share of the batch. tp = 0 takes the widest split that
    `shard_ranges` accepts and that divides `world` (GPT-2-124M on 8 ranks: 2 groups of 4)."""
    if world < 1:
        raise ValueError(f"{world} ranks")
    if tp:
        if world % tp or not splits(config, tp):
            raise ValueError(f"{world} ranks do not form groups of {tp} tensor-parallel ranks")
        return world // tp, tp
    best = max(t for t in range(1, world + 1) if world % t == 0 and splits(config, t))
    return world // best, best


def hybrid_groups(tp: int):
    """(group, dp_index): this rank's tensor-parallel group -- ranks [i * tp, (i + 1) * tp) form
    group i -- and i. Every rank creates every group, in the same order, as
    torch.distributed.new_group requires; with tp equal to the world the group is the world."""
    import torch.distributed as dist

    world, rank = dist.get_world_size(), dist.get_rank()
    if world % tp:
        raise ValueError(f"{world} ranks do not form groups of {tp}")
    if tp == world:
        return dist.group.WORLD, 0
    mine = None
    for i in range(world // tp):
        ranks = list(range(i * tp, (i + 1) * tp))
        group = dist.new_group(ranks)
        if rank in ranks:
            mine = group
    return mine, rank // tp


def shard_block(blk: dict, config: Config, shard: TPShard) -> dict:
    """This rank's weights of one block (torch tensors on any device; [out, in] layouts):
    w_qkv/b_qkv the local q, k, v heads side by side; w_o the local input columns; w_fc/b_fc
    the local hidden units; w_proj the local input columns. Biases of the row-parallel layers
    stay whole (rank 0 adds them once)."""
    import torch

    c, d = config.width, config.head_dim
    h0, h1 = shard.heads
    f0, f1 = shard.hidden
    cols = slice(h0 * d, h1 * d)
    parts = [slice(i * c + h0 * d, i * c + h1 * d) for i in range(3)]
    return {
        "ln1_g": blk["ln1_g"], "ln1_b": blk["ln1_b"],
        "w_qkv": torch.cat([blk["w_qkv"][p] for p in parts]).contiguous(),
        "b_qkv": torch.cat([blk["b_qkv"][p] for p in parts]).contiguous(),
        "w_o": blk["w_o"][:, cols].contiguous(), "b_o": blk["b_o"],
        "ln2_g": blk["ln2_g"], "ln2_b": blk["ln2_b"],
        "w_fc": blk["w_fc"][f0:f1].contiguous(), "b_fc": blk["b_fc"][f0:f1].contiguous(),
        "w_proj": blk["w_proj"][:, f0:f1].contiguous(), "b_proj": blk["b_proj"],
    }


class GPT2TensorParallel:
    """This rank's part of a randomly initialised GPT-2 (the same weights as GPT2(config, seed)
    on every rank, then sliced). Call forward on every rank of `group` with the same ids."""

    def __init__(self, config: Config = GPT2_124M, seed: int = 0, group=None,
                 exchange: str = "nccl") -> None:
        import torch
        import torch.distributed as dist

        if exchange not in ("nccl", "nvlink"):
            raise ValueError(f"exchange {exchange!r}: 'nccl' or 'nvlink'")
        self.config = config
        self.group = group
        self.exchange = exchange
        self._nvlink: dict | None = None
        self._epoch = 0
        rank = dist.get_rank(group) if dist.is_initialized() else 0
        size = dist.get_world_size(group) if dist.is_initialized() else 1
        self.shard = shard_ranges(config, rank, size)
        full = GPT2(config, seed)
        self.wte, self.wpe = full.wte, full.wpe
        v0, v1 = self.shard.vocab
        self.head = full.wte[v0:v1].contiguous()
        self.blocks = [shard_block(b, config, self.shard) for b in full.blocks]
        self.lnf_g, self.lnf_b = full.lnf_g, full.lnf_b
        self.layernorm = full.layernorm
        self.lib = runtime.library()
        _bind(self.lib)
        _bind_exchange(self.lib)
        self._buffers: dict = {}
        del full
        torch.cuda.empty_cache()

    def _scratch(self, tokens: int):
        import torch

        found = self._buffers.get(tokens)
        if found is None:
            c, d = self.config.width, "cuda"
            hl = self.shard.heads[1] - self.shard.heads[0]
            wl = hl * self.config.head_dim
            fl = self.shard.hidden[1] - self.shard.hidden[0]
            found = {
                "x": torch.empty(tokens, c, dtype=torch.float32, device=d),
                "h": torch.empty(tokens, c, dtype=torch.bfloat16, device=d),
                "qkv": torch.empty(tokens, 3 * wl, dtype=torch.bfloat16, device=d),
                "vt": torch.empty(tokens * wl, dtype=torch.bfloat16, device=d),
                "att": torch.empty(tokens, wl, dtype=torch.bfloat16, device=d),
                "f": torch.empty(tokens, fl, dtype=torch.bfloat16, device=d),
                "status": torch.zeros(1, dtype=torch.int32, device=d),
            }
            self._buffers = {tokens: found}
        return found

    def _check(self, status: int, what: str) -> None:
        if status != runtime.STATUS_OK:
            raise runtime.B200Error(f"{what}: {runtime.last_error()}")

    # ---------------------------------------------------------------- the NVLink exchange

    def _exchange_state(self, tokens: int) -> dict:
        """Exchange buffers for `tokens` rows and the flag arrays: this rank's, and every other
        rank's mapped here. Made by all ranks of the group together. One allocation per rank:
        the exchange buffer (two parities x one [ceil(tokens / size), width] f32 slot per rank,
        the partials of this rank's row block), then the gather buffer (the same shape: the
        other ranks' summed blocks). The flag array holds the first round's flags at [0, 8)
        and the second's at [8, 16)."""
        import torch.distributed as dist

        if self._nvlink is not None and self._nvlink["tokens"] == tokens:
            return self._nvlink
        self.close()
        lib, size, rank = self.lib, self.shard.size, self.shard.rank
        block_rows = -(-tokens // size)
        slot = block_rows * self.config.width
        handle = (ctypes.c_uint8 * 64)()
        flag_handle = (ctypes.c_uint8 * 64)()
        own = lib.ppyb200_shared_alloc(2 * 2 * size * slot * 4, handle)
        flags = lib.ppyb200_shared_alloc(64, flag_handle)
        if not own or not flags:
            raise runtime.B200Error(f"exchange buffers: {runtime.last_error()}")
        gathered = [None] * size
        dist.all_gather_object(gathered, (bytes(handle), bytes(flag_handle)), group=self.group)
        buffers, flag_arrays = [], []
        for s, (bh, fh) in enumerate(gathered):
            if s == rank:
                buffers.append(own)
                flag_arrays.append(flags)
                continue
            mapped = lib.ppyb200_shared_open((ctypes.c_uint8 * 64).from_buffer_copy(bh))
            mapped_flags = lib.ppyb200_shared_open((ctypes.c_uint8 * 64).from_buffer_copy(fh))
            if not mapped or not mapped_flags:
                raise runtime.B200Error(f"rank {s}'s exchange buffers: {runtime.last_error()}")
            buffers.append(mapped)
            flag_arrays.append(mapped_flags)
        self._epoch = 0  # the flags start at 0
        self._nvlink = {"tokens": tokens, "slot": slot, "own": own, "flags": flags,
                        "buffers": buffers, "flag_arrays": flag_arrays,
                        "first": (ctypes.c_void_p * size)(*flag_arrays),
                        "second": (ctypes.c_void_p * size)(*[f + 32 for f in flag_arrays])}
        return self._nvlink

    def close(self) -> None:
        """Unmap the other ranks' exchange buffers and free this rank's (all ranks together:
        a barrier sits between the two)."""
        import torch
        import torch.distributed as dist

        state, self._nvlink = self._nvlink, None
        if state is None:
            return
        torch.cuda.synchronize()
        for s, (buffer, flags) in enumerate(zip(state["buffers"], state["flag_arrays"])):
            if s != self.shard.rank:
                self.lib.ppyb200_shared_close(buffer)
                self.lib.ppyb200_shared_close(flags)
        dist.barrier(group=self.group)
        self.lib.ppyb200_shared_free(state["own"])
        self.lib.ppyb200_shared_free(state["flags"])

    def _row_parallel_nvlink(self, a, w, bias, x, tokens, k, st, what):
        """The reduce-scatter form: partials of row block s to rank s, the owner sums its block
        and sends it to every rank (csrc/tp_exchange.cu)."""
        state = self._exchange_state(tokens)
        size, rank, slot = self.shard.size, self.shard.rank, state["slot"]
        self._epoch += 1
        epoch, parity = self._epoch, self._epoch & 1
        c = self.config.width
        exchange = 4 * parity * size * slot            # byte offsets in each rank's allocation
        gather = 4 * (2 + parity) * size * slot
        # this rank's slot, in parity `parity`, of every rank's exchange and gather buffers
        slots = (ctypes.c_void_p * size)(
            *[b + exchange + 4 * rank * slot for b in state["buffers"]])
        peers = (ctypes.c_void_p * size)(
            *[b + gather + 4 * rank * slot for b in state["buffers"]])
        lib = self.lib
        self._check(lib.ppyb200_tp_partial_reduce_scatter(a.data_ptr(), w.data_ptr(), slots,
                                                          size, tokens, c, k, st), what)
        self._check(lib.ppyb200_tp_signal(state["first"], size, rank, epoch), what)
        self._check(lib.ppyb200_tp_reduce_block(x.data_ptr(), bias.data_ptr(),
                                                state["own"] + exchange, peers, state["flags"],
                                                size, rank, tokens, c, epoch, st), what)
        self._check(lib.ppyb200_tp_signal(state["second"], size, rank, epoch), what)
        self._check(lib.ppyb200_tp_gather_blocks(x.data_ptr(), state["own"] + gather,
                                                 state["flags"] + 32, size, rank, tokens, c,
                                                 epoch, st), what)

    def _row_parallel(self, a, w, bias, x, tokens, k, st, what):
        """x <- x + bias + sum over ranks of a_r @ w_r^T (rank 0 keeps x and the bias)."""
        import torch.distributed as dist

        if self.exchange == "nvlink" and self.shard.size > 1:
            self._row_parallel_nvlink(a, w, bias, x, tokens, k, st, what)
            return
        c = self.config.width
        if self.shard.rank == 0:
            status = self.lib.ppyb200_linear_residual(a.data_ptr(), w.data_ptr(), bias.data_ptr(),
                                                      x.data_ptr(), tokens, c, k, st)
        else:
            status = self.lib.ppyb200_matmul_bf16_kmajor(a.data_ptr(), w.data_ptr(), None,
                                                         x.data_ptr(), tokens, c, k)
        self._check(status, what)
        if self.shard.size > 1:
            dist.all_reduce(x, group=self.group)

    def new_logits(self, batch: int, length: int):
        """This rank's f32 [batch, length, v1 - v0] logits with rows on 128-byte lines (the
        row pitch rounded up to 32 floats), as GPT2.new_logits."""
        import torch

        v0, v1 = self.shard.vocab
        pitch = (v1 - v0 + 31) // 32 * 32
        rows = torch.empty(batch, length, pitch, dtype=torch.float32, device="cuda")
        return rows[:, :, :v1 - v0]

    def forward(self, ids, logits=None):
        """This rank's logits [batch, length, v1 - v0] (f32) for the vocab rows [v0, v1),
        into `logits` when given (any evenly spaced rows), else into new_logits()."""
        cfg = self.config
        batch, length = ids.shape
        tokens = batch * length
        c = cfg.width
        hl = self.shard.heads[1] - self.shard.heads[0]
        wl = hl * cfg.head_dim
        fl = self.shard.hidden[1] - self.shard.hidden[0]
        v0, v1 = self.shard.vocab
        if length > cfg.context or length % 128 != 0:
            raise runtime.B200Error("the sequence length is a multiple of 128 up to the context")
        ids = ids.contiguous()
        s = self._scratch(tokens)
        x, h, qkv, vt, att, f = s["x"], s["h"], s["qkv"], s["vt"], s["att"], s["f"]
        status = s["status"]
        if logits is None:
            logits = self.new_logits(batch, length)
        pitch = GPT2._row_pitch(logits, batch, length, v1 - v0)
        lib = self.lib
        st = status.data_ptr()
        status.zero_()
        self._check(lib.ppyb200_gpt2_embed(ids.data_ptr(), self.wte.data_ptr(),
                                           self.wpe.data_ptr(), x.data_ptr(), tokens, length, c,
                                           cfg.vocab, st), "embed")
        ln = self.layernorm.device.layernorm_bf16
        for blk in self.blocks:
            self._check(ln(x, blk["ln1_g"], blk["ln1_b"], h).status, "layernorm")
            self._check(lib.ppyb200_linear_qkv_bf16(h.data_ptr(), blk["w_qkv"].data_ptr(),
                                                    blk["b_qkv"].data_ptr(), qkv.data_ptr(),
                                                    vt.data_ptr(), tokens, c, length, hl, st),
                        "qkv")
            self._check(lib.ppyb200_attention_causal_vt_bf16(qkv.data_ptr(), vt.data_ptr(),
                                                             att.data_ptr(), batch, length, hl,
                                                             cfg.head_dim, st), "attention")
            self._row_parallel(att, blk["w_o"], blk["b_o"], x, tokens, wl, st, "out projection")
            self._check(ln(x, blk["ln2_g"], blk["ln2_b"], h).status, "layernorm")
            self._check(lib.ppyb200_linear_bf16(h.data_ptr(), blk["w_fc"].data_ptr(),
                                                blk["b_fc"].data_ptr(), f.data_ptr(), tokens, fl,
                                                c, 1, st), "fc")
            self._row_parallel(f, blk["w_proj"], blk["b_proj"], x, tokens, fl, st, "proj")
        self._check(ln(x, self.lnf_g, self.lnf_b, h).status, "layernorm")
        self._check(lib.ppyb200_matmul_bf16_kmajor_ld(h.data_ptr(), self.head.data_ptr(), None,
                                                      logits.data_ptr(), pitch, tokens, v1 - v0,
                                                      c), "lm head")
        return logits

    def status(self) -> int:
        for buffers in self._buffers.values():
            return int(buffers["status"].item())
        return 0
