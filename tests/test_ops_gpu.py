"""GPU parity: every hot-path op through the C ABI against the CPU oracle.

Tolerances (the north star's): fp32 paths <= 1e-4, bf16 tensor-core paths with
f32 accumulate <= 2e-2 (max abs error normalised by max(1, max |ref|));
int8 quantise / dequantise, argmax, embedding: bit-exact.
"""
import math

import numpy as np
import pytest

from gpu_util import (BF16_TOL, F32_TOL, assert_close, bf16_round, dev, no_device_error, np_of, rng,
                      to_gpu, torch)
from golden_io import load

import oracle

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _gpu():
    dev()
    yield
    no_device_error()


def ops():
    from teenygrad_b200 import ops as o
    return o


# ------------------------------------------------------------------ norms --
def test_rmsnorm_golden_f32():
    x = load("rmsnorm", "x.bin", (16, 128))
    w = load("rmsnorm", "weight.bin")
    y, rrms = ops().rms_norm(to_gpu(x), to_gpu(w), eps=1e-8, return_rrms=True)
    assert_close(np_of(y), load("rmsnorm", "expected_forward.bin", (16, 128)), F32_TOL)
    assert_close(np_of(rrms), load("rmsnorm", "expected_rrms.bin"), F32_TOL)


@pytest.mark.parametrize("M,N", [(16, 2048), (257, 2048), (3, 129), (128, 256)])
def test_rmsnorm_bf16(M, N):
    r = rng(M + N)
    x = bf16_round(r.standard_normal((M, N)))
    w = bf16_round(r.uniform(0.5, 1.5, N))
    ref, rr = oracle.rmsnorm(x, w, 1e-5)
    y, rrms = ops().rms_norm(to_gpu(x, torch.bfloat16), to_gpu(w, torch.bfloat16), eps=1e-5, return_rrms=True)
    assert_close(np_of(y), ref, BF16_TOL)
    assert_close(np_of(rrms), rr, 1e-5)


def test_layernorm_golden_and_bf16():
    x = load("layernorm", "x.bin", (16, 128))
    y = ops().layer_norm(to_gpu(x), to_gpu(load("layernorm", "weight.bin")), to_gpu(load("layernorm", "bias.bin")), 1e-5)
    assert_close(np_of(y), load("layernorm", "expected_forward.bin", (16, 128)), F32_TOL)
    r = rng(5)
    x = bf16_round(r.standard_normal((300, 2048)) * 3 + 1)
    w, b = bf16_round(r.uniform(0.5, 1.5, 2048)), bf16_round(r.normal(0, 0.1, 2048))
    ref = oracle.layernorm(x, w, b, 1e-5)
    y = ops().layer_norm(*(to_gpu(a, torch.bfloat16) for a in (x, w, b)), 1e-5)
    assert_close(np_of(y), ref, BF16_TOL)


# ------------------------------------------------------------ elementwise --
@pytest.mark.parametrize("name,kind,tol", [("silu", "silu", 1e-5), ("gelu", "gelu_tanh", 2e-5),
                                           ("relu", "relu", 0.0), ("sigmoid", "sigmoid", 1e-5)])
def test_activation_golden(name, kind, tol):
    x = load(name, "x.bin")
    y = ops().activation(kind, to_gpu(x))
    np.testing.assert_allclose(np_of(y), load(name, "expected_forward.bin"), atol=tol, rtol=0)


@pytest.mark.parametrize("n", [1, 7, 1000003])
def test_elementwise_bf16_and_tails(n):
    r = rng(n)
    a = bf16_round(r.standard_normal(n) * 3)
    b = bf16_round(r.standard_normal(n))
    for kind in ("silu", "gelu_tanh", "relu", "sigmoid"):
        y = ops().activation(kind, to_gpu(a, torch.bfloat16))
        assert_close(np_of(y), oracle.act(kind, a), BF16_TOL, kind)
    assert_close(np_of(ops().swiglu(to_gpu(a, torch.bfloat16), to_gpu(b, torch.bfloat16))), oracle.swiglu(a, b), BF16_TOL)
    assert_close(np_of(ops().add(to_gpu(a, torch.bfloat16), to_gpu(b, torch.bfloat16))), oracle.add(a, b), BF16_TOL)
    af = a.astype(np.float32)
    assert_close(np_of(ops().swiglu(to_gpu(af), to_gpu(b))), oracle.swiglu(af, b), F32_TOL)
    np.testing.assert_array_equal(np_of(ops().add(to_gpu(af), to_gpu(b))), oracle.add(af, b))


# ----------------------------------------------------------------- linear --
def test_linear_golden_f32():
    x = load("linear", "input.bin", (64, 64))
    w = load("linear", "weight.bin", (48, 64))
    b = load("linear", "bias.bin")
    y0 = ops().linear(to_gpu(x), to_gpu(w))
    y1 = ops().linear(to_gpu(x), to_gpu(w), bias=to_gpu(b))
    exp0 = load("linear", "expected_no_bias.bin", (64, 48))
    exp1 = load("linear", "expected_with_bias.bin", (64, 48))
    # values reach |y| ~ 300: relative 1e-4
    assert_close(np_of(y0) / 300, exp0 / 300, F32_TOL)
    assert_close(np_of(y1) / 300, exp1 / 300, F32_TOL)


@pytest.mark.parametrize("M,N,K", [(128, 768, 256), (128, 256, 1024), (37, 50, 3)])
def test_linear_f32(M, N, K):
    r = rng(M * N + K)
    x = r.standard_normal((M, K)).astype(np.float32)
    w = (r.standard_normal((N, K)) * 0.02).astype(np.float32)
    res = r.standard_normal((M, N)).astype(np.float32)
    y = ops().linear(to_gpu(x), to_gpu(w), residual=to_gpu(res))
    assert_close(np_of(y), oracle.linear(x, w, resid=res), F32_TOL)


@pytest.mark.parametrize("M,N,K", [(256, 384, 512), (200, 264, 520), (1000, 1024, 2048), (129, 128, 64)])
def test_linear_bf16_tc(M, N, K):
    r = rng(M + N + K)
    x = bf16_round(r.standard_normal((M, K)))
    w = bf16_round(r.standard_normal((N, K)) * 0.02)
    bias = r.standard_normal(N).astype(np.float32) * 0.1
    res = bf16_round(r.standard_normal((M, N)))
    xg, wg = to_gpu(x, torch.bfloat16), to_gpu(w, torch.bfloat16)
    assert_close(np_of(ops().linear(xg, wg)), oracle.linear(x, w), BF16_TOL, "plain")
    y = ops().linear(xg, wg, bias=to_gpu(bias), residual=to_gpu(res, torch.bfloat16))
    assert_close(np_of(y), oracle.linear(x, w, bias, res), BF16_TOL, "bias+res")
    y32 = ops().linear(xg, wg, out_f32=True)
    assert y32.dtype == torch.float32
    assert_close(np_of(y32), oracle.linear(x, w), 2e-3, "f32 out")


@pytest.mark.parametrize("M", [256, 1, 16, 64])
def test_linear_bf16_swiglu(M):
    r = rng(M)
    K, F = 512, 512
    x = bf16_round(r.standard_normal((M, K)))
    wg = bf16_round(r.standard_normal((F, K)) * 0.05)
    wu = bf16_round(r.standard_normal((F, K)) * 0.05)
    W = ops().interleave_gate_up(to_gpu(wg, torch.bfloat16), to_gpu(wu, torch.bfloat16))
    y = ops().linear(to_gpu(x, torch.bfloat16), W, swiglu=True)
    ref = oracle.swiglu(oracle.linear(x, wg), oracle.linear(x, wu))
    assert y.shape == (M, F)
    assert_close(np_of(y), ref, BF16_TOL)


@pytest.mark.parametrize("M,N,K", [(1, 3072, 2048), (16, 2048, 2048), (24, 2048, 2048), (33, 1000, 512), (64, 32000, 2048),
                                   (16, 2048, 8192)])
def test_linear_bf16_decode_gemv(M, N, K):
    r = rng(M * 7 + N)
    x = bf16_round(r.standard_normal((M, K)))
    w = bf16_round(r.standard_normal((N, K)) * 0.02)
    res = bf16_round(r.standard_normal((M, N)))
    y = ops().linear(to_gpu(x, torch.bfloat16), to_gpu(w, torch.bfloat16), residual=to_gpu(res, torch.bfloat16))
    assert_close(np_of(y), oracle.linear(x, w, resid=res), BF16_TOL)
    # twice in a row: split-K counters must be back at zero
    y2 = ops().linear(to_gpu(x, torch.bfloat16), to_gpu(w, torch.bfloat16), residual=to_gpu(res, torch.bfloat16))
    assert torch.equal(y, y2)


def test_linear_padded_output_rows_f32():
    # the reference executor gives LinearForward an output whose rows are padded to 16
    # bytes (N = 6 f32 -> stride 8) and the kernel writes only the first N columns
    r = rng(21)
    x = r.standard_normal((64, 64)).astype(np.float32)
    w = r.standard_normal((6, 64)).astype(np.float32)
    b = r.standard_normal(6).astype(np.float32)
    buf, y = ops().linear_padded(to_gpu(x), to_gpu(w), to_gpu(b))
    assert buf.shape == (64, 8)
    assert_close(np_of(y), oracle.linear(x, w, b), F32_TOL)
    assert torch.isnan(buf[:, 6:]).all()


@pytest.mark.parametrize("M", [16, 256])
def test_linear_strided_bf16(M):
    # x rows read from a wider buffer (ldx > K), y rows written into a wider one
    # (ldy > N): the decode GEMV (M = 16) and the tensor-core GEMM (M = 256)
    from teenygrad_b200 import _lib
    import ctypes
    r = rng(M + 5)
    K, N, ldx, ldy = 256, 48, 320, 64
    xw = bf16_round(r.standard_normal((M, ldx)))
    w = bf16_round(r.standard_normal((N, K)) * 0.05)
    bias = r.standard_normal(N).astype(np.float32)
    xg = to_gpu(xw, torch.bfloat16)
    wg = to_gpu(w, torch.bfloat16)
    bg = to_gpu(bias)
    y = torch.full((M, ldy), 7.0, device="cuda", dtype=torch.bfloat16)
    ctx = ops().context()
    _lib.check(ctx, _lib.lib().tb_linear_fwd_strided(ctx, 1, ctypes.c_void_p(xg.data_ptr()), ctypes.c_int64(ldx),
                                                     ctypes.c_void_p(wg.data_ptr()), ctypes.c_void_p(bg.data_ptr()),
                                                     None, ctypes.c_void_p(y.data_ptr()), ctypes.c_int64(ldy),
                                                     ctypes.c_int64(M), ctypes.c_int64(N), ctypes.c_int64(K),
                                                     ctypes.c_int(1)))
    torch.cuda.synchronize()
    assert_close(np_of(y[:, :N]), oracle.linear(xw[:, :K], w, bias), BF16_TOL)
    assert (y[:, N:] == 7.0).all()


def test_matmul():
    r = rng(11)
    a = r.standard_normal((70, 96)).astype(np.float32)
    b = r.standard_normal((96, 40)).astype(np.float32)
    assert_close(np_of(ops().matmul(to_gpu(a), to_gpu(b))), oracle.matmul(a, b), F32_TOL)
    a = bf16_round(r.standard_normal((300, 512)))
    b = bf16_round(r.standard_normal((512, 264)) * 0.05)
    got = ops().matmul(to_gpu(a, torch.bfloat16), to_gpu(b, torch.bfloat16))
    assert_close(np_of(got), oracle.matmul(a, b), BF16_TOL)


# ------------------------------------------------------------------- int8 --
def test_quantize_int8_bit_exact():
    r = rng(3)
    w = (r.standard_normal((513, 700)) * 0.02).astype(np.float32)
    w[0] = 0.0
    w[1, :5] = [0.5, -0.5, 1.5, -2.5, 127.0]
    w[2, 0] = -0.0
    # non-finite weights follow Rust's saturating `as i32` (affine.rs:101-139):
    # NaN -> 0; a row with -Inf gets scale 1; a row with +Inf gets scale Inf
    w[3, 7] = np.nan
    w[4, 2] = -np.inf
    w[5, 3] = np.inf
    w[6, 1:3] = [np.inf, np.nan]
    w[7, :] = np.nan
    w[8, 0] = 1e30
    q, s = ops().quantize_int8(to_gpu(w))
    qo, so = oracle.quantize_int8(w)
    np.testing.assert_array_equal(q.cpu().numpy(), qo)
    np.testing.assert_array_equal(s.cpu().numpy(), so)
    qn, sn = oracle.quantize_int8_numpy(w)
    np.testing.assert_array_equal(qo, qn)
    assert qo[3, 7] == 0 and so[4] == 1.0 and qo[4, 2] == -127 and np.isinf(so[5]) and qo[5, 3] == 0
    assert not qo[7].any() and so[7] == 1.0
    deq = ops().dequantize_int8(q, s)
    np.testing.assert_array_equal(deq.cpu().numpy(), oracle.dequantize_int8(qo, so))
    # bf16 weights (upcast exactly)
    wb = bf16_round(w)
    qb, sb = ops().quantize_int8(to_gpu(wb, torch.bfloat16))
    qo, so = oracle.quantize_int8(wb)
    np.testing.assert_array_equal(qb.cpu().numpy(), qo)
    np.testing.assert_array_equal(sb.cpu().numpy(), so)


@pytest.mark.parametrize("M,N,K", [(64, 2048, 2048), (16, 3072, 2048), (1, 2048, 8192), (64, 1000, 512),
                                   (16, 256, 48), (64, 512, 320), (24, 1024, 1536)])
def test_int8_linear(M, N, K):
    r = rng(M + N + K)
    w = (r.standard_normal((N, K)) * 0.02).astype(np.float32)
    q, s = oracle.quantize_int8(w)
    x = bf16_round(r.standard_normal((M, K)))
    res = bf16_round(r.standard_normal((M, N)))
    y = ops().int8_linear(to_gpu(x, torch.bfloat16), to_gpu(q, torch.int8), to_gpu(s), residual=to_gpu(res, torch.bfloat16))
    assert_close(np_of(y), oracle.int8_linear(x, q, s, resid=res), BF16_TOL)


@pytest.mark.parametrize("M", [16, 64])
def test_int8_linear_every_byte_exact(M):
    # q[n, k] runs through all 256 byte values (-128 included); one-hot token rows pick
    # column k = m, so y[m, n] = q[n, m] * 1.0 exactly in bf16: checks the int8 -> bf16
    # weight conversion bit for bit
    N, K = 256, 256
    n, k = np.meshgrid(np.arange(N), np.arange(K), indexing="ij")
    q = (((n + 3 * k) % 256) - 128).astype(np.int8)
    s = np.ones(N, np.float32)
    x = np.zeros((M, K), np.float32)
    x[np.arange(M), np.arange(M)] = 1.0
    y = ops().int8_linear(to_gpu(x, torch.bfloat16), to_gpu(q, torch.int8), to_gpu(s))
    got = np_of(y)
    np.testing.assert_array_equal(got, q[:, :M].T.astype(np.float32))
    np.testing.assert_array_equal(got, oracle.int8_linear(x, q, s))


def test_int8_linear_swiglu():
    r = rng(9)
    M, K, F = 64, 1024, 512
    wg = (r.standard_normal((F, K)) * 0.05).astype(np.float32)
    wu = (r.standard_normal((F, K)) * 0.05).astype(np.float32)
    W = ops().interleave_gate_up(torch.from_numpy(wg), torch.from_numpy(wu)).numpy()
    q, s = oracle.quantize_int8(W)
    x = bf16_round(r.standard_normal((M, K)))
    y = ops().int8_linear(to_gpu(x, torch.bfloat16), to_gpu(q, torch.int8), to_gpu(s), swiglu=True)
    full = oracle.int8_linear(x, q, s).reshape(M, F // 128, 2, 128)
    ref = oracle.swiglu(full[:, :, 0, :].reshape(M, F), full[:, :, 1, :].reshape(M, F))
    assert_close(np_of(y), ref, BF16_TOL)


# -------------------------------------------------------------- attention --
def test_attention_golden_f32():
    q = load("flash_attn2", "q.bin", (1, 4, 8, 64))
    k = load("flash_attn2", "k.bin", (1, 4, 8, 64))
    v = load("flash_attn2", "v.bin", (1, 4, 8, 64))
    o, lse = ops().attention(to_gpu(q), to_gpu(k), to_gpu(v), scale=0.125, return_lse=True)
    assert_close(np_of(o), load("flash_attn2", "expected_forward_o.bin", (1, 4, 8, 64)), F32_TOL)
    assert_close(np_of(lse), load("flash_attn2", "expected_forward_l.bin", (1, 4, 8)), F32_TOL)


def test_attention_f32_causal_gqa():
    r = rng(4)
    q = r.standard_normal((1, 4, 128, 64)).astype(np.float32)
    k = r.standard_normal((1, 2, 128, 64)).astype(np.float32)
    v = r.standard_normal((1, 2, 128, 64)).astype(np.float32)
    o, lse = ops().attention(to_gpu(q), to_gpu(k), to_gpu(v), scale=0.125, causal=True, return_lse=True)
    ro, rl = oracle.attention(q, k, v, 0.125, True)
    assert_close(np_of(o), ro, F32_TOL)
    assert_close(np_of(lse), rl, F32_TOL)


@pytest.mark.parametrize("B,Hq,Hkv,Sq,Sk,D,causal", [
    (1, 2, 2, 128, 128, 64, False),
    (1, 4, 2, 300, 300, 64, True),
    (2, 4, 1, 256, 256, 128, True),
    (1, 2, 2, 200, 456, 128, True),
    (1, 2, 2, 130, 77, 64, False),
    (1, 4, 2, 300, 200, 128, False),
])
def test_attention_bf16_tc(B, Hq, Hkv, Sq, Sk, D, causal):
    r = rng(B * 1000 + Sq + Sk + D)
    q = bf16_round(r.standard_normal((B, Hq, Sq, D)))
    k = bf16_round(r.standard_normal((B, Hkv, Sk, D)))
    v = bf16_round(r.standard_normal((B, Hkv, Sk, D)))
    sc = 1.0 / math.sqrt(D)
    o, lse = ops().attention(*(to_gpu(a, torch.bfloat16) for a in (q, k, v)), scale=sc, causal=causal, return_lse=True)
    ro, rl = oracle.attention(q, k, v, sc, causal)
    assert_close(np_of(o), ro, BF16_TOL, "O")
    assert_close(np_of(lse), rl, 1e-3, "LSE")


# The benchmarked shapes: a slice of C3 (causal prefill, S 4096, D 128, 2 of its
# 256 (batch, head) pairs) and C4 prefill (GQA 32 / 8 heads, D 64, S 1024, 2 of
# its 16 sequences), each with O and LSE against the oracle.
@pytest.mark.parametrize("B,Hq,Hkv,S,D", [(1, 2, 2, 4096, 128), (2, 32, 8, 1024, 64)])
def test_attention_bf16_benchmark_shapes(B, Hq, Hkv, S, D):
    r = rng(S + D)
    q = bf16_round(r.standard_normal((B, Hq, S, D)))
    k = bf16_round(r.standard_normal((B, Hkv, S, D)))
    v = bf16_round(r.standard_normal((B, Hkv, S, D)))
    sc = 1.0 / math.sqrt(D)
    o, lse = ops().attention(*(to_gpu(a, torch.bfloat16) for a in (q, k, v)), scale=sc, causal=True, return_lse=True)
    ro, rl = oracle.attention(q, k, v, sc, True)
    assert_close(np_of(o), ro, BF16_TOL, "O")
    assert_close(np_of(lse), rl, 1e-3, "LSE")


@pytest.mark.parametrize("D", [64, 128])
def test_attention_causal_rows_without_keys(D):
    # causal with Sq > Sk (bottom-right aligned): the first Sq - Sk queries see no key, so
    # whole query tiles have no key tile at all; O is 0 and LSE -inf there, as in the oracle
    r = rng(D + 7)
    B, Hq, Hkv, Sq, Sk = 1, 2, 1, 300, 100
    q = bf16_round(r.standard_normal((B, Hq, Sq, D)))
    k = bf16_round(r.standard_normal((B, Hkv, Sk, D)))
    v = bf16_round(r.standard_normal((B, Hkv, Sk, D)))
    sc = 1.0 / math.sqrt(D)
    o, lse = ops().attention(*(to_gpu(a, torch.bfloat16) for a in (q, k, v)), scale=sc, causal=True, return_lse=True)
    ro, rl = oracle.attention(q, k, v, sc, True)
    assert_close(np_of(o), ro, BF16_TOL, "O")
    got = np_of(lse)
    masked = np.isneginf(rl)
    assert masked.any() and not masked.all()
    assert np.array_equal(np.isneginf(got), masked), "LSE -inf pattern"
    assert_close(got[~masked], rl[~masked], 1e-3, "LSE")


# (16, 32, 8, 1100, 64) is the C4 decode shape: two splits of five 128-key tiles, three
# tile pairs per split with the last one short.
@pytest.mark.parametrize("B,Hq,Hkv,Sk,D", [(4, 32, 8, 1000, 64), (2, 8, 8, 2048, 128), (3, 4, 1, 5, 64),
                                           (16, 32, 8, 1100, 64)])
def test_attention_decode(B, Hq, Hkv, Sk, D):
    r = rng(Sk + D)
    q = bf16_round(r.standard_normal((B, Hq, 1, D)))
    k = bf16_round(r.standard_normal((B, Hkv, Sk, D)))
    v = bf16_round(r.standard_normal((B, Hkv, Sk, D)))
    sc = 1.0 / math.sqrt(D)
    o, lse = ops().attention(*(to_gpu(a, torch.bfloat16) for a in (q, k, v)), scale=sc, causal=True, return_lse=True)
    ro, rl = oracle.attention(q, k, v, sc, True)
    assert_close(np_of(o), ro, BF16_TOL, "O")
    assert_close(np_of(lse), rl, 1e-3, "LSE")


@pytest.mark.parametrize("pos", [200, 700, 1050])
def test_attention_decode_late_max(pos):
    """A key far more aligned with the queries than the rest, at a late position: the
    split that holds it raises its reference max (and rescales O and the row sums) on
    the tile pair of that key, after earlier pairs were accumulated."""
    B, Hq, Hkv, Sk, D = 4, 32, 8, 1100, 64
    r = rng(pos)
    q = bf16_round(r.standard_normal((B, Hq, 1, D)))
    k = bf16_round(r.standard_normal((B, Hkv, Sk, D)))
    v = bf16_round(r.standard_normal((B, Hkv, Sk, D)))
    G = Hq // Hkv
    for g in range(Hkv):   # key pos of group g points along its first query head
        k[:, g, pos, :] = bf16_round(q[:, g * G, 0, :] * 1.5)
    sc = 1.0 / math.sqrt(D)
    o, lse = ops().attention(*(to_gpu(a, torch.bfloat16) for a in (q, k, v)), scale=sc, causal=True, return_lse=True)
    ro, rl = oracle.attention(q, k, v, sc, True)
    assert_close(np_of(o), ro, BF16_TOL, "O")
    assert_close(np_of(lse), rl, 1e-3, "LSE")


# ---------------------------------------------------------- decoder pieces --
def test_rope_embedding_argmax():
    r = rng(8)
    x = bf16_round(r.standard_normal((40, 8, 64)))
    pos = r.integers(0, 2048, 40).astype(np.int32)
    y = ops().rope(to_gpu(x, torch.bfloat16), to_gpu(pos, torch.int32))
    assert_close(np_of(y), oracle.rope(x, pos, 10000.0), BF16_TOL)
    table = bf16_round(r.standard_normal((1000, 256)))
    ids = r.integers(0, 1000, 77).astype(np.int32)
    e = ops().embedding(to_gpu(table, torch.bfloat16), to_gpu(ids, torch.int32))
    np.testing.assert_array_equal(np_of(e), oracle.embedding(table, ids))
    logits = r.standard_normal((16, 32000)).astype(np.float32)
    logits[3, 100] = logits[3, 200] = 50.0            # tie -> lower index
    logits[5, :] = -np.inf
    logits[7, 10] = np.nan
    got = ops().argmax(to_gpu(logits)).cpu().numpy()
    np.testing.assert_array_equal(got, oracle.argmax(logits))
    assert got[3] == 100
