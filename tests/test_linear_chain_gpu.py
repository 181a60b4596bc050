"""tb_linear_chain_fwd: dependent decode linear layers in one persistent launch.

Each chain mirrors a decoder layer's decode GEMVs: the output projection with
its residual, gate/up with the RMSNorm fused in front and SwiGLU, down with its
residual, then a projection of the new residual stream with the norm fused.
The reference composes the oracle's rmsnorm / linear / swiglu in f32 from the
same bf16 inputs, rounding each stored intermediate to bf16 as the chain
stores it.  Tolerance: bf16 (2e-2, normalised max abs error).  The split-K
reduction sums in a fixed order, so two runs agree bit for bit.
"""
import numpy as np
import pytest

from gpu_util import BF16_TOL, assert_close, bf16_round, dev, no_device_error, np_of, rng, to_gpu, torch
import oracle

pytestmark = pytest.mark.gpu


def _interleave(gate, up):
    from teenygrad_b200 import ops
    return ops.interleave_gate_up(gate, up)


def _case(M, d, f, q_out, seed):
    """Inputs of one chain: attention output a [M, d], residual stream h [M, d]."""
    g = rng(seed)
    t = lambda *s, sc=1.0: bf16_round(g.standard_normal(s).astype(np.float32) * sc)  # noqa: E731
    return dict(a=t(M, d), h=t(M, d), wo=t(d, d, sc=0.03), gate=t(f, d, sc=0.03), up=t(f, d, sc=0.03),
                wd=t(d, f, sc=0.02), wq=t(q_out, d, sc=0.03), g1=t(d, sc=0.5) + 1, g2=t(d, sc=0.5) + 1)


def _reference(c, eps):
    h = bf16_round(oracle.linear(c["a"], c["wo"], resid=c["h"]))
    n = oracle.rmsnorm(h, c["g1"], eps)[0]
    act = bf16_round(oracle.swiglu(oracle.linear(n, c["gate"]), oracle.linear(n, c["up"])))
    h2 = bf16_round(oracle.linear(act, c["wd"], resid=h))
    q = bf16_round(oracle.linear(oracle.rmsnorm(h2, c["g2"], eps)[0], c["wq"]))
    return h2, act, q


def _run(c, eps, n_steps=4):
    from teenygrad_b200 import ops
    bf = torch.bfloat16
    a, h = to_gpu(c["a"], bf), to_gpu(c["h"], bf)
    wo, wd, wq = to_gpu(c["wo"], bf), to_gpu(c["wd"], bf), to_gpu(c["wq"], bf)
    wgu = _interleave(to_gpu(c["gate"], bf), to_gpu(c["up"], bf))
    g1, g2 = to_gpu(c["g1"], bf), to_gpu(c["g2"], bf)
    M, f = a.shape[0], c["gate"].shape[0]
    act = torch.empty(M, f, device=a.device, dtype=bf)
    q = torch.empty(M, wq.shape[0], device=a.device, dtype=bf)
    steps = [dict(x=a, w=wo, y=h, residual=h),
             dict(x=h, w=wgu, y=act, norm_w=g1, eps=eps, swiglu=True),
             dict(x=act, w=wd, y=h, residual=h),
             dict(x=h, w=wq, y=q, norm_w=g2, eps=eps)][:n_steps]
    ops.linear_chain(steps)
    torch.cuda.synchronize()
    return np_of(h), np_of(act), np_of(q)


# (M, d_model, ffn, last projection rows): the C4 layer shape at batch 16, a small
# model (few CTAs, every tile shared), odd token counts, the 64-token tile
@pytest.mark.parametrize("M,d,f,qn", [(16, 2048, 8192, 3072), (3, 256, 512, 512), (1, 512, 1024, 768),
                                      (29, 1024, 2048, 1536), (64, 512, 1536, 1024)])
def test_linear_chain_matches_oracle(M, d, f, qn):
    dev()
    eps = 1e-5
    c = _case(M, d, f, qn, seed=M + d)
    h2, act, q = _run(c, eps)
    r_h2, r_act, r_q = _reference(c, eps)
    assert_close(act, r_act, BF16_TOL, "gate/up (norm + SwiGLU)")
    assert_close(h2, r_h2, BF16_TOL, "down + residual")
    assert_close(q, r_q, BF16_TOL, "projection (norm)")
    no_device_error()


def test_linear_chain_deterministic_and_partial():
    dev()
    c = _case(16, 2048, 8192, 3072, seed=5)
    first = _run(c, 1e-5)
    again = _run(c, 1e-5)
    for x, y in zip(first, again):
        assert np.array_equal(x, y)
    # a one-step chain is the output projection alone
    from teenygrad_b200 import ops
    h1 = _run(c, 1e-5, n_steps=1)[0]
    ref = np_of(ops.linear(to_gpu(c["a"], torch.bfloat16), to_gpu(c["wo"], torch.bfloat16),
                           residual=to_gpu(c["h"], torch.bfloat16)))
    assert_close(h1, ref, BF16_TOL, "one step vs tb_linear_fwd")
    no_device_error()


def test_linear_chain_rejects_bad_steps():
    dev()
    from teenygrad_b200 import ops
    bf = torch.bfloat16
    x = torch.zeros(4, 256, device="cuda", dtype=bf)
    y = torch.zeros(4, 200, device="cuda", dtype=bf)
    with pytest.raises(RuntimeError):
        ops.linear_chain([dict(x=x, w=torch.zeros(200, 256, device="cuda", dtype=bf), y=y)])   # N % 256
    with pytest.raises(RuntimeError):
        big = torch.zeros(65, 256, device="cuda", dtype=bf)
        ops.linear_chain([dict(x=big, w=torch.zeros(256, 256, device="cuda", dtype=bf), y=big)])   # M > 64
    with pytest.raises(RuntimeError):
        ops.linear_chain([dict(x=x, w=torch.zeros(256, 256, device="cuda", dtype=bf), y=x)] * 5)   # > 4 steps
    no_device_error()
