"""The graph executor (tb_graph_*) and the lowering of recorded ops onto it:
the C1 block, a bf16 token pipeline (Gather -> RmsNorm -> Linear ->
RotaryEmbedding -> ArgMax) and a conv stage, each against the oracle."""
import math

import numpy as np
import pytest

import oracle
from gpu_util import BF16_TOL, F32_TOL, assert_close, bf16_round, dev, no_device_error, np_of, rng, to_gpu, torch
from oracle.decoder import block_forward as oracle_block

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("capture", [True, False])
def test_graph_c1_block(capture):
    dev()
    from teenygrad_b200.block import block_graph, random_block_params
    p = random_block_params(seed=3)
    g = block_graph(p, 1, 128, 4, 1e-6, capture=capture)
    pn = {k: v.cpu().numpy() for k, v in p.items()}
    for seed in (1, 2):   # a second run replays the captured graph on new input
        x = torch.randn(1, 128, 256, generator=torch.Generator().manual_seed(seed)).cuda()
        (y,) = g.run(x)
        torch.cuda.synchronize()
        assert_close(np_of(y), oracle_block(x.cpu().numpy(), pn, 4, 1e-6), F32_TOL)
    # intermediates share the arena: it is smaller than all of them side by side
    # x, h, qkv, o, x1, h2, gate, up, swiglu, y side by side
    inter = 4 * 128 * (256 + 256 + 768 + 256 + 256 + 256 + 3 * 1024 + 256)
    assert g.arena_bytes() < 0.8 * inter
    no_device_error()


def test_graph_bf16_token_pipeline():
    dev()
    from teenygrad_b200.graph import Graph
    r = rng(31)
    V, d, H, D, T = 512, 256, 4, 64, 24
    table = bf16_round(r.standard_normal((V, d)))
    w = bf16_round(r.uniform(0.8, 1.2, d))
    Wq = bf16_round(r.standard_normal((H * D, d)) * 0.05)
    Wl = bf16_round(r.standard_normal((V, d)) * 0.05)
    ids = r.integers(0, V, T).astype(np.int32)
    pos = np.arange(T, dtype=np.int32) + 5
    g = Graph()
    gi, gp = g.input((T,), torch.int32), g.input((T,), torch.int32)
    x = g.gather(g.param(to_gpu(table, torch.bfloat16)), gi)
    h = g.rms_norm(x, g.param(to_gpu(w, torch.bfloat16)), 1e-5)
    q = g.linear(h, g.param(to_gpu(Wq, torch.bfloat16)))
    logits = g.linear(h, g.param(to_gpu(Wl, torch.bfloat16)))
    am = g.argmax(logits)
    g.output(q, logits, am)
    g.compile(capture=True)
    q_o, lg, am_o = g.run(torch.from_numpy(ids), torch.from_numpy(pos))
    torch.cuda.synchronize()
    xr = oracle.embedding(table, ids)
    hr = bf16_round(oracle.rmsnorm(xr, w, 1e-5)[0])
    assert_close(np_of(q_o), oracle.linear(hr, Wq), BF16_TOL, "q")
    lref = oracle.linear(hr, Wl)
    assert_close(np_of(lg), lref, BF16_TOL, "logits")
    np.testing.assert_array_equal(am_o.cpu().numpy(), oracle.argmax(np_of(lg)))
    no_device_error()


@pytest.mark.parametrize("dtype,Hq,Hkv,D", [(torch.float32, 4, 2, 32), (torch.bfloat16, 8, 2, 64),
                                            (torch.bfloat16, 2, 2, 128)])
def test_graph_attention_token_major(dtype, Hq, Hkv, D):
    # separate projections: q [B, S, Hq D], k / v [B, S, Hkv D], read in place
    dev()
    from teenygrad_b200.graph import Graph
    r = rng(Hq + D)
    B, S = 2, 200
    cast = bf16_round if dtype == torch.bfloat16 else (lambda a: np.asarray(a, np.float32))
    q = cast(r.standard_normal((B, S, Hq * D)))
    k = cast(r.standard_normal((B, S, Hkv * D)))
    v = cast(r.standard_normal((B, S, Hkv * D)))
    g = Graph()
    gq, gk, gv = g.input(q.shape, dtype), g.input(k.shape, dtype), g.input(v.shape, dtype)
    g.output(g.multi_head_attention(gq, gk, gv, heads=Hq, kv_heads=Hkv, causal=True))
    g.compile(capture=True)
    (o,) = g.run(*(to_gpu(a, dtype) for a in (q, k, v)))
    torch.cuda.synchronize()
    heads = lambda a, H: a.reshape(B, S, H, D).transpose(0, 2, 1, 3)
    ro, _ = oracle.attention(heads(q, Hq), heads(k, Hkv), heads(v, Hkv), 1.0 / math.sqrt(D), True)
    ref = ro.transpose(0, 2, 1, 3).reshape(B, S, Hq * D)
    assert_close(np_of(o), ref, BF16_TOL if dtype == torch.bfloat16 else F32_TOL)
    no_device_error()


def test_graph_rope_node():
    dev()
    from teenygrad_b200.graph import Graph
    r = rng(32)
    x = bf16_round(r.standard_normal((40, 8, 64)))
    pos = r.integers(0, 2048, 40).astype(np.int32)
    g = Graph()
    gx, gp = g.input((40, 8, 64), torch.bfloat16), g.input((40,), torch.int32)
    y = g.rotary_embedding(gx, gp, theta=10000.0)
    g.output(y)
    g.compile(capture=False)
    (yo,) = g.run(to_gpu(x, torch.bfloat16), torch.from_numpy(pos))
    torch.cuda.synchronize()
    assert_close(np_of(yo), oracle.rope(x, pos, 10000.0), BF16_TOL)


def test_graph_conv_stage_bf16():
    dev()
    from teenygrad_b200.graph import Graph
    r = rng(33)
    B, C, Hh = 4, 64, 24
    x = bf16_round(r.standard_normal((B, C, Hh, Hh)))
    ws = [bf16_round(r.standard_normal((C, C, 3, 3)) * math.sqrt(2 / (C * 9))) for _ in range(2)]
    sc = [r.uniform(0.5, 1.5, C).astype(np.float32) for _ in range(2)]
    sh = [(r.standard_normal(C) * 0.1).astype(np.float32) for _ in range(2)]
    g = Graph()
    y = gx = g.input((B, C, Hh, Hh), torch.bfloat16)
    for i in range(2):
        y = g.conv2d(y, g.param(to_gpu(ws[i], torch.bfloat16)), None, g.param(to_gpu(sc[i])), g.param(to_gpu(sh[i])),
                     stride=1, pad=1, act="relu")
    g.output(y)
    g.compile(capture=True)
    (yo,) = g.run(to_gpu(x, torch.bfloat16))
    torch.cuda.synchronize()
    ref = x
    for i in range(2):
        ref = bf16_round(oracle.conv2d(ref, ws[i], scale=sc[i], shift=sh[i], pad=1, act="relu"))
    assert_close(np_of(yo), ref, BF16_TOL)
    no_device_error()


def test_graph_lowering_errors():
    dev()
    from teenygrad_b200 import TeenyError
    from teenygrad_b200.graph import Graph
    g = Graph()
    a, b = g.input((4, 8)), g.input((4, 8))
    g.output(g.mul(a, b))                 # Mul lowers only as Mul(Silu(gate), up)
    with pytest.raises(TeenyError):
        g.compile()
    g2 = Graph()
    x = g2.input((4, 8))
    with pytest.raises(TeenyError):
        g2.linear(x, g2.param(torch.zeros(16, 7, device="cuda")))   # K mismatch: caught when lowered
        g2.compile()
