"""ORACLE -- test infrastructure only: GPT-2's forward in float32 torch.

The reference's GPT-2 path is a torch ATen region (examples/46_gpt2/gpt2.ppy:18-57 for a
block, :210-241 for the forward): layernorm, a QKV linear, causal scaled-dot-product
attention, the output projection and residual, layernorm, the GELU-tanh MLP and residual,
a final layernorm and the tied head `normed @ wte.T`. This module restates it with torch's
own f32 operators, on the weights of a ppy_b200 GPT2 model (`forward`) or on a fresh CPU
copy of the same seeded initialisation (`cpu_model`). The parity tests, the smoke check and
bench.py's CPU-baseline leg use it; nothing under ppy_b200/ imports it.
"""

from __future__ import annotations


def forward(model, ids):
    """Logits [batch, length, vocab] in float32 for token ids [batch, length], computed by
    torch on `model`'s device from the model's (bf16) weights taken as f32."""
    import torch.nn.functional as F

    cfg = model.config
    batch, length = ids.shape
    c, heads, hd = cfg.width, cfg.heads, cfg.head_dim
    x = model.wte.float()[ids] + model.wpe.float()[:length]
    for blk in model.blocks:
        hh = F.layer_norm(x, (c,), blk["ln1_g"], blk["ln1_b"], 1e-5)
        qkv = F.linear(hh, blk["w_qkv"].float(), blk["b_qkv"])
        q, k, v = qkv.split(c, dim=-1)
        q = q.reshape(batch, length, heads, hd).transpose(1, 2)
        k = k.reshape(batch, length, heads, hd).transpose(1, 2)
        v = v.reshape(batch, length, heads, hd).transpose(1, 2)
        a = F.scaled_dot_product_attention(q, k, v, is_causal=True)
        a = a.transpose(1, 2).reshape(batch, length, c)
        x = x + F.linear(a, blk["w_o"].float(), blk["b_o"])
        n = F.layer_norm(x, (c,), blk["ln2_g"], blk["ln2_b"], 1e-5)
        ff = F.gelu(F.linear(n, blk["w_fc"].float(), blk["b_fc"]), approximate="tanh")
        x = x + F.linear(ff, blk["w_proj"].float(), blk["b_proj"])
    n = F.layer_norm(x, (c,), model.lnf_g, model.lnf_b, 1e-5)
    return n @ model.wte.float().t()


def cpu_model(seed: int = 0, layers: int = 12):
    """A callable ids -> logits: GPT-2-124M on the CPU in float32, with the weights of a
    ppy_b200 GPT2(seed=seed) drawn the same way (N(0, 0.02), rounded to bf16 as the GPU model
    keeps them; zero biases, unit layernorm gains). The reference's own path on host cores."""
    import torch
    import torch.nn.functional as F

    g = torch.Generator().manual_seed(seed)
    c, v, heads, context = 768, 50257, 12, 1024

    def normal(*shape):
        return (0.02 * torch.randn(*shape, generator=g)).to(torch.bfloat16).float()

    wte, wpe = normal(v, c), normal(context, c)
    blocks = [(normal(3 * c, c), normal(c, c), normal(4 * c, c), normal(c, 4 * c))
              for _ in range(layers)]
    ones, zeros = torch.ones(c), torch.zeros(c)

    def run(ids):
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

    return run
