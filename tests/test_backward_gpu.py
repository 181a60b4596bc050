"""GPU parity of the backward kernels against the reference's golden vectors
(flash_attn2, linear, conv2d / conv2d_padded backward fixtures) and the CPU
oracle (causal / GQA attention, RMSNorm, bf16, strided conv).

Tolerances: f32 <= 1e-4 (normalised max abs error), bf16 <= 2e-2."""
import math

import numpy as np
import pytest

import oracle
from golden_io import load
from gpu_util import BF16_TOL, F32_TOL, assert_close, bf16_round, dev, no_device_error, np_of, rng, to_gpu, torch

pytestmark = pytest.mark.gpu


def ops():
    dev()
    from teenygrad_b200 import ops as o
    return o


def test_attention_bwd_golden_f32():
    sh = (1, 4, 8, 64)
    q, k, v = (load("flash_attn2", f, sh) for f in ("q.bin", "k.bin", "v.bin"))
    o = load("flash_attn2", "expected_forward_o.bin", sh)
    lse = load("flash_attn2", "expected_forward_l.bin", (1, 4, 8))
    do = load("flash_attn2", "do.bin", sh)
    dq, dk, dv = ops().attention_backward(*(to_gpu(a) for a in (q, k, v, o, do, lse)), scale=0.125)
    assert_close(np_of(dq), load("flash_attn2", "expected_backward_dq.bin", sh), F32_TOL, "dq")
    assert_close(np_of(dk), load("flash_attn2", "expected_backward_dk.bin", sh), F32_TOL, "dk")
    assert_close(np_of(dv), load("flash_attn2", "expected_backward_dv.bin", sh), F32_TOL, "dv")
    no_device_error()


@pytest.mark.parametrize("dtype,B,Hq,Hkv,Sq,Sk,D,causal", [
    (torch.float32, 2, 4, 2, 70, 70, 64, True),
    (torch.float32, 1, 4, 1, 33, 100, 128, True),
    (torch.float32, 1, 2, 2, 50, 40, 64, False),
    (torch.bfloat16, 1, 8, 2, 130, 130, 64, True),
])
def test_attention_bwd_vs_oracle(dtype, B, Hq, Hkv, Sq, Sk, D, causal):
    r = rng(Sq + Sk + D)
    cast = bf16_round if dtype == torch.bfloat16 else (lambda a: np.asarray(a, np.float32))
    q = cast(r.standard_normal((B, Hq, Sq, D)))
    k = cast(r.standard_normal((B, Hkv, Sk, D)))
    v = cast(r.standard_normal((B, Hkv, Sk, D)))
    do = cast(r.standard_normal((B, Hq, Sq, D)))
    sc = 1.0 / math.sqrt(D)
    o, lse = oracle.attention(q, k, v, sc, causal)
    o = cast(o)
    rq, rk, rv = oracle.attention_bwd(q, k, v, o, do, lse, sc, causal)
    g = lambda a: to_gpu(a, dtype)
    dq, dk, dv = ops().attention_backward(g(q), g(k), g(v), g(o), g(do), to_gpu(lse), scale=sc, causal=causal)
    tol = BF16_TOL if dtype == torch.bfloat16 else F32_TOL
    assert_close(np_of(dq), rq, tol, "dq")
    assert_close(np_of(dk), rk, tol, "dk")
    assert_close(np_of(dv), rv, tol, "dv")
    no_device_error()


def test_linear_bwd_golden_f32():
    x = load("linear", "input.bin", (64, 64))
    w = load("linear", "weight.bin", (48, 64))
    dy = load("linear", "dy.bin", (64, 48))
    dx, dw, db = ops().linear_backward(to_gpu(x), to_gpu(w), to_gpu(dy))
    assert_close(np_of(dx), load("linear", "expected_dx.bin", (64, 64)), F32_TOL, "dx")
    assert_close(np_of(dw), load("linear", "expected_dw.bin", (48, 64)), F32_TOL, "dw")
    assert_close(np_of(db), load("linear", "expected_db.bin", (48,)), F32_TOL, "db")
    no_device_error()


@pytest.mark.parametrize("M,N,K", [(256, 512, 384), (64, 2048, 256), (1000, 136, 72)])
def test_linear_bwd_bf16_vs_oracle(M, N, K):
    r = rng(M + N + K)
    x = bf16_round(r.standard_normal((M, K)))
    w = bf16_round(r.standard_normal((N, K)) * 0.05)
    dy = bf16_round(r.standard_normal((M, N)))
    rx, rw, rb = oracle.linear_bwd(x, w, dy)
    dx, dw, db = ops().linear_backward(to_gpu(x, torch.bfloat16), to_gpu(w, torch.bfloat16), to_gpu(dy, torch.bfloat16))
    assert_close(np_of(dx), rx, BF16_TOL, "dx")
    assert_close(np_of(dw), rw, BF16_TOL, "dw")
    assert_close(np_of(db), rb, 1e-4, "db")
    no_device_error()


@pytest.mark.parametrize("name,pad,oh", [("conv2d", 0, 6), ("conv2d_padded", 1, 8)])
def test_conv2d_bwd_golden_f32(name, pad, oh):
    x = load(name, "x.bin", (1, 2, 8, 8))
    w = load(name, "w.bin", (4, 2, 3, 3))
    dy = load(name, "dy.bin", (1, 4, oh, oh))
    dx, dw = ops().conv2d_backward(to_gpu(dy), to_gpu(x), to_gpu(w), 1, pad)
    assert_close(np_of(dx), load(name, "expected_dx.bin", (1, 2, 8, 8)), F32_TOL, "dx")
    assert_close(np_of(dw), load(name, "expected_dw.bin", (4, 2, 3, 3)), F32_TOL, "dw")
    no_device_error()


@pytest.mark.parametrize("dtype,B,Cin,Cout,H,W,K,stride,pad", [
    (torch.float32, 2, 3, 5, 11, 9, 3, 2, 1),
    (torch.float32, 4, 16, 8, 14, 14, 5, 1, 2),
    (torch.bfloat16, 2, 64, 64, 28, 28, 3, 1, 1),
])
def test_conv2d_bwd_vs_oracle(dtype, B, Cin, Cout, H, W, K, stride, pad):
    r = rng(B + Cin + H)
    cast = bf16_round if dtype == torch.bfloat16 else (lambda a: np.asarray(a, np.float32))
    x = cast(r.standard_normal((B, Cin, H, W)))
    w = cast(r.standard_normal((Cout, Cin, K, K)) * 0.1)
    OH = (H + 2 * pad - K) // stride + 1
    OW = (W + 2 * pad - K) // stride + 1
    dy = cast(r.standard_normal((B, Cout, OH, OW)))
    rx, rw = oracle.conv2d_bwd(dy, x, w, stride, pad)
    dx, dw = ops().conv2d_backward(to_gpu(dy, dtype), to_gpu(x, dtype), to_gpu(w, dtype), stride, pad)
    tol = BF16_TOL if dtype == torch.bfloat16 else F32_TOL
    assert_close(np_of(dx), rx, tol, "dx")
    assert_close(np_of(dw), rw, tol, "dw")
    no_device_error()


@pytest.mark.parametrize("dtype,M,N", [(torch.float32, 16, 128), (torch.float32, 300, 2048),
                                       (torch.bfloat16, 1024, 2048)])
def test_rmsnorm_bwd_vs_oracle(dtype, M, N):
    r = rng(M + N)
    cast = bf16_round if dtype == torch.bfloat16 else (lambda a: np.asarray(a, np.float32))
    x = cast(r.uniform(-2, 2, (M, N)))
    w = cast(r.uniform(0.5, 1.5, N))
    dy = cast(r.uniform(-1, 1, (M, N)))
    _, rrms = oracle.rmsnorm(x, w, 1e-6)
    dw0 = r.standard_normal(N).astype(np.float32)
    rdx, rdw = oracle.rmsnorm_bwd(dy, x, w, rrms, dw0)
    dx, dw = ops().rms_norm_backward(to_gpu(dy, dtype), to_gpu(x, dtype), to_gpu(w, dtype), to_gpu(rrms), to_gpu(dw0))
    tol = BF16_TOL if dtype == torch.bfloat16 else F32_TOL
    assert_close(np_of(dx), rdx, tol, "dx")
    assert_close(np_of(dw), rdw, 1e-4, "dw")
    # deterministic: a second run gives the same bits
    dx2, dw2 = ops().rms_norm_backward(to_gpu(dy, dtype), to_gpu(x, dtype), to_gpu(w, dtype), to_gpu(rrms), to_gpu(dw0))
    assert torch.equal(dx, dx2) and torch.equal(dw, dw2)
    no_device_error()
