"""Pre-norm transformer block from the library's ops.

x -> x + Wo attn(rmsnorm(x))  -> x + Wd (silu(Wg h) * (Wu h)), h = rmsnorm(x)

fp32 end to end (f32 CUDA-core linear and attention paths), causal SDPA with
scale 1/sqrt(head_dim), no RoPE (the config names none).  The reference has
no block-level op; this is the composition its graph would lower to from
RmsNorm / Linear / attention / SiLU / Mul / Add nodes
(kernels/teeny-kernels/src/graph/mod.rs:1117, :1228, :1734).

block_graph() records exactly those ops on a Graph and compiles it onto the
library's graph executor: planned buffers, native kernels only (the head
split of the attention is a library kernel), one CUDA graph per run.
block_forward() is the same composition op by op.
"""
from __future__ import annotations

import math

import torch

from . import ops


def block_forward(x, p, n_heads, eps=1e-6):
    """x [B, S, d] f32; p: dict of f32 cuda tensors attn_norm [d], wq/wk/wv/wo
    [d, d], mlp_norm [d], w_gate/w_up [F, d], w_down [d, F]."""
    B, S, d = x.shape
    hd = d // n_heads
    h = ops.rms_norm(x, p["attn_norm"], eps)
    # one projection GEMM for q, k and v: rows of wq, wk, wv stacked (each output
    # element is the same dot product as with the separate weights)
    wqkv = p.get("wqkv")
    if wqkv is None:
        wqkv = torch.cat([p["wq"], p["wk"], p["wv"]], 0)
    q, k, v = ops.linear(h, wqkv).split(d, dim=-1)

    def heads(t):
        return t.view(B, S, n_heads, hd).transpose(1, 2).contiguous()

    o = ops.attention(heads(q), heads(k), heads(v), scale=1.0 / math.sqrt(hd), causal=True)
    o = o.transpose(1, 2).contiguous().view(B, S, d)
    x = ops.linear(o, p["wo"], residual=x)
    h = ops.rms_norm(x, p["mlp_norm"], eps)
    a = ops.swiglu(ops.linear(h, p["w_gate"]), ops.linear(h, p["w_up"]))
    return ops.linear(a, p["w_down"], residual=x)


def block_graph(p, B, S, n_heads, eps=1e-6, capture=True):
    """The block as a compiled Graph (teenygrad_b200.graph): input x [B, S, d] f32,
    output y [B, S, d].  Run with g.run(x) or, on an input already written, g.launch()."""
    from .graph import Graph
    d = p["wq"].shape[1]
    g = Graph()
    x = g.input((B, S, d))
    if "wqkv" not in p:
        p = dict(p, wqkv=torch.cat([p["wq"], p["wk"], p["wv"]], 0))
    P = {k: g.param(v) for k, v in p.items() if k not in ("wq", "wk", "wv")}
    h = g.rms_norm(x, P["attn_norm"], eps)
    qkv = g.linear(h, P["wqkv"])      # one projection; attention reads q, k, v from it in place
    o = g.multi_head_attention(qkv, heads=n_heads, causal=True, scale=1.0 / math.sqrt(d // n_heads))
    x1 = g.linear(o, P["wo"], residual=x)
    h2 = g.rms_norm(x1, P["mlp_norm"], eps)
    a = g.mul(g.silu(g.linear(h2, P["w_gate"])), g.linear(h2, P["w_up"]))   # lowers to one SwiGLU node
    y = g.linear(a, P["w_down"], residual=x1)
    g.output(y)
    return g.compile(capture=capture)


def random_block_params(d=256, F=1024, seed=0, device="cuda"):
    g = torch.Generator(device="cpu").manual_seed(seed)

    def w(*s):
        return (torch.randn(*s, generator=g) * 0.02).to(device)

    p = dict(attn_norm=torch.ones(d, device=device), wq=w(d, d), wk=w(d, d), wv=w(d, d), wo=w(d, d),
             mlp_norm=torch.ones(d, device=device), w_gate=w(F, d), w_up=w(F, d), w_down=w(d, F))
    p["wqkv"] = torch.cat([p["wq"], p["wk"], p["wv"]], 0)
    return p
