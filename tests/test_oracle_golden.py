"""Pin the CPU oracle to the reference's own golden vectors.

Tolerances are the reference tests' own: 1e-4 for rmsnorm / layernorm /
flash_attn2 / conv2d (test_rmsnorm.rs:144, test_layernorm.rs:159,
test_flash_attn2.rs:165, test_conv2d_bias.rs:232), 2e-5 for gelu
(test_gelu.rs:108), 1e-5 for the sigmoid family (test_sigmoid.rs:129).
"""
import hashlib
import os

import numpy as np
import pytest

import oracle
from golden_io import GOLDEN, load


def test_manifest_hashes():
    lines = [l.split() for l in open(os.path.join(GOLDEN, "MANIFEST.txt")) if not l.startswith("#")]
    assert len(lines) >= 40
    for rel, size, sha in lines:
        data = open(os.path.join(GOLDEN, rel), "rb").read()
        assert len(data) == int(size)
        assert hashlib.sha256(data).hexdigest() == sha, rel


def test_rmsnorm_golden():
    x = load("rmsnorm", "x.bin", (16, 128))
    w = load("rmsnorm", "weight.bin")
    y, rrms = oracle.rmsnorm(x, w, 1e-8)
    np.testing.assert_allclose(y, load("rmsnorm", "expected_forward.bin", (16, 128)), atol=1e-4, rtol=0)
    np.testing.assert_allclose(rrms, load("rmsnorm", "expected_rrms.bin"), atol=1e-4, rtol=0)


def test_layernorm_golden():
    x = load("layernorm", "x.bin", (16, 128))
    y = oracle.layernorm(x, load("layernorm", "weight.bin"), load("layernorm", "bias.bin"), 1e-5)
    np.testing.assert_allclose(y, load("layernorm", "expected_forward.bin", (16, 128)), atol=1e-4, rtol=0)


@pytest.mark.parametrize("name,kind,tol", [("silu", "silu", 1e-5), ("gelu", "gelu_tanh", 2e-5),
                                           ("relu", "relu", 0.0), ("sigmoid", "sigmoid", 1e-5)])
def test_activation_golden(name, kind, tol):
    x = load(name, "x.bin")
    np.testing.assert_allclose(oracle.act(kind, x), load(name, "expected_forward.bin"), atol=tol, rtol=0)


def test_add_mul_golden():
    a, b = load("elemwise_add", "a.bin"), load("elemwise_add", "b.bin")
    np.testing.assert_array_equal(oracle.add(a, b), load("elemwise_add", "expected_fwd.bin"))
    a, b = load("elemwise_binary", "a.bin"), load("elemwise_binary", "b.bin")
    # SwiGLU's product half: elemwise_mul_forward.
    one = np.full_like(a, 1e30)  # silu(1e30) == 1e30 exactly -> swiglu(g, u) = g*u check below
    np.testing.assert_allclose(a * b, load("elemwise_binary", "expected_mul.bin"), rtol=1e-6)
    del one


def test_linear_golden():
    x = load("linear", "input.bin", (64, 64))
    w = load("linear", "weight.bin", (48, 64))
    b = load("linear", "bias.bin")
    # test_linear.rs:48-55 uses TF32 tolerances; the exact oracle meets 1e-4 relative.
    np.testing.assert_allclose(oracle.linear(x, w), load("linear", "expected_no_bias.bin", (64, 48)),
                               atol=1e-3, rtol=1e-5)
    np.testing.assert_allclose(oracle.linear(x, w, b), load("linear", "expected_with_bias.bin", (64, 48)),
                               atol=1e-3, rtol=1e-5)


@pytest.mark.parametrize("name,pad,oh", [("conv2d", 0, 6), ("conv2d_padded", 1, 8)])
def test_conv2d_golden(name, pad, oh):
    x = load(name, "x.bin", (1, 2, 8, 8))
    w = load(name, "w.bin", (4, 2, 3, 3))
    y = oracle.conv2d(x, w, stride=1, pad=pad)
    np.testing.assert_allclose(y, load(name, "expected_forward.bin", (1, 4, oh, oh)), atol=1e-4, rtol=0)


def test_batchnorm_golden():
    x = load("batchnorm", "x.bin", (64, 32))
    y = oracle.batchnorm_inference(x, load("batchnorm", "weight.bin"), load("batchnorm", "bias.bin"),
                                   load("batchnorm", "running_mean.bin"),
                                   load("batchnorm", "running_var.bin"), 1e-5)
    np.testing.assert_allclose(y, load("batchnorm", "expected_forward_inference.bin", (64, 32)),
                               atol=1e-4, rtol=0)


def test_bn_fold_matches_batchnorm():
    rng = np.random.default_rng(1)
    x = rng.standard_normal((2, 3, 5, 5)).astype(np.float32)
    w = rng.standard_normal((4, 3, 3, 3)).astype(np.float32) * 0.2
    bias = rng.standard_normal(4).astype(np.float32)
    g, be = rng.uniform(0.5, 1.5, 4), rng.normal(0, 0.1, 4)
    mu, var = rng.normal(0, 0.1, 4), rng.uniform(0.5, 1.5, 4)
    sc, sh = oracle.bn_fold(g, be, mu, var, 1e-5, bias)
    fused = oracle.conv2d(x, w, scale=sc, shift=sh, pad=1, act="relu")
    plain = oracle.conv2d(x, w, bias=bias, pad=1)
    bn = oracle.batchnorm_inference(plain, g, be, mu, var, 1e-5)
    np.testing.assert_allclose(fused, np.maximum(bn, 0), atol=1e-5)


def test_flash_attn2_golden():
    q = load("flash_attn2", "q.bin", (1, 4, 8, 64))
    k = load("flash_attn2", "k.bin", (1, 4, 8, 64))
    v = load("flash_attn2", "v.bin", (1, 4, 8, 64))
    o, lse = oracle.attention(q, k, v, 1.0 / 8.0, causal=False)
    np.testing.assert_allclose(o, load("flash_attn2", "expected_forward_o.bin", (1, 4, 8, 64)), atol=1e-4, rtol=0)
    np.testing.assert_allclose(lse, load("flash_attn2", "expected_forward_l.bin", (1, 4, 8)), atol=1e-4, rtol=0)


def test_attention_causal_gqa_vs_torch():
    torch = pytest.importorskip("torch")
    rng = np.random.default_rng(3)
    q = rng.standard_normal((2, 8, 33, 64)).astype(np.float32)
    k = rng.standard_normal((2, 2, 33, 64)).astype(np.float32)
    v = rng.standard_normal((2, 2, 33, 64)).astype(np.float32)
    o, lse = oracle.attention(q, k, v, 0.125, causal=True)
    kt = torch.from_numpy(k).repeat_interleave(4, dim=1)
    vt = torch.from_numpy(v).repeat_interleave(4, dim=1)
    ref = torch.nn.functional.scaled_dot_product_attention(torch.from_numpy(q), kt, vt, is_causal=True, scale=0.125)
    np.testing.assert_allclose(o, ref.numpy(), atol=1e-5)
    s = torch.from_numpy(q) @ kt.transpose(-1, -2) * 0.125
    s = s.masked_fill(torch.triu(torch.ones(33, 33, dtype=torch.bool), 1), float("-inf"))
    np.testing.assert_allclose(lse, torch.logsumexp(s, -1).numpy(), atol=1e-5)


def test_quantize_int8_c_vs_numpy():
    rng = np.random.default_rng(7)
    w = (rng.standard_normal((257, 300)) * 0.02).astype(np.float32)
    w[3] = 0.0                                   # amax == 0 row -> scale 1
    w[5, :4] = [0.5, -0.5, 1.5, -2.5]            # exact .5 ties after scaling
    w[5, 4] = 127.0 * 2.5 / 127.0
    w[6, 0] = -0.0
    q, s = oracle.quantize_int8(w)
    qn, sn = oracle.quantize_int8_numpy(w)
    np.testing.assert_array_equal(q, qn)
    np.testing.assert_array_equal(s, sn)
    assert s[3] == 1.0 and not q[3].any()
    assert q.min() >= -127 and q.max() <= 127
    # round-trip tolerance of quant/affine.rs tests: |deq - w| <= scale / 2
    deq = oracle.dequantize_int8(q, s)
    assert np.all(np.abs(deq - w) <= s[:, None] * 0.5 + 1e-12)


def test_quantize_int8_non_finite():
    # Rust semantics (affine.rs:91-139): NaN fails every comparison, so the
    # min/max pass skips it; a row holding -Inf has a non-finite minimum and
    # gets scale 1; a row holding +Inf gets scale Inf; `round() as i32`
    # saturates (NaN -> 0, +-Inf -> i32 limits) before the clamp.
    w = np.full((6, 5), 0.25, np.float32)
    w[0, 1] = np.nan
    w[1, 2] = -np.inf
    w[2, 3] = np.inf
    w[3, :] = np.nan
    w[4, 0], w[4, 1] = np.inf, np.nan
    w[5, 0] = 3e38
    q, s = oracle.quantize_int8(w)
    qn, sn = oracle.quantize_int8_numpy(w)
    np.testing.assert_array_equal(q, qn)
    np.testing.assert_array_equal(s, sn)
    assert q[0].tolist() == [127, 0, 127, 127, 127]
    assert s[1] == 1.0 and q[1].tolist() == [0, 0, -127, 0, 0]
    assert np.isinf(s[2]) and q[2].tolist() == [0, 0, 0, 0, 0]
    assert s[3] == 1.0 and not q[3].any()
    assert np.isinf(s[4]) and q[4].tolist() == [0, 0, 0, 0, 0]
    assert q[5, 0] == 127 and q[5, 1] == 0


def test_quantize_half_away_from_zero():
    # amax = 2.54 -> scale = 0.02; 0.01/0.02 = 0.5 exactly representable? use
    # a scale of 1 row (amax = 127) so x/scale = x and ties are exact.
    w = np.array([[127.0, 0.5, -0.5, 1.5, -1.5, 2.5, -2.5, 0.49999997]], np.float32)
    q, s = oracle.quantize_int8(w)
    assert s[0] == 1.0
    assert q.tolist() == [[127, 1, -1, 2, -2, 3, -3, 0]]


def test_rope_and_argmax():
    x = np.random.default_rng(0).standard_normal((3, 2, 8)).astype(np.float32)
    y = oracle.rope(x, np.array([0, 1, 5], np.int32), 10000.0)
    np.testing.assert_allclose(y[0], x[0], atol=1e-7)          # position 0 is identity
    np.testing.assert_allclose(np.linalg.norm(y, axis=-1), np.linalg.norm(x, axis=-1), rtol=1e-5)
    a = np.array([[1, 3, 3, 2], [-np.inf, -np.inf, -np.inf, -np.inf], [0, np.nan, 5, 5]], np.float32)
    assert oracle.argmax(a).tolist() == [1, 0, 2]


def test_bf16_rounding():
    x = np.array([1.0, 1.00390625, 1.01171875, -3.0e38, 1e-40], np.float32)
    bits = oracle.bf16_bits(x)
    assert bits[0] == 0x3F80
    assert bits[1] == 0x3F80          # tie -> even
    assert bits[2] == 0x3F82          # tie -> even (up)
    t = pytest.importorskip("torch")
    r = t.from_numpy(np.random.default_rng(0).standard_normal(4096).astype(np.float32))
    np.testing.assert_array_equal(oracle.round_bf16(r.numpy()), r.bfloat16().float().numpy())


# ---------------------------------------------------------------- backward --
def _rel(got, ref):
    return float(np.abs(got - ref).max()) / max(1.0, float(np.abs(ref).max()))


def test_attention_bwd_oracle_golden():
    # fixtures: BH 4, N 8, HD 64, non-causal (generate.py:701-747); tolerance of test_flash_attn2.rs
    sh = (1, 4, 8, 64)
    q, k, v = (load("flash_attn2", f, sh) for f in ("q.bin", "k.bin", "v.bin"))
    o = load("flash_attn2", "expected_forward_o.bin", sh)
    lse = load("flash_attn2", "expected_forward_l.bin", (1, 4, 8))
    do = load("flash_attn2", "do.bin", sh)
    dq, dk, dv = oracle.attention_bwd(q, k, v, o, do, lse, 0.125, False)
    assert _rel(dq, load("flash_attn2", "expected_backward_dq.bin", sh)) < 1e-4
    assert _rel(dk, load("flash_attn2", "expected_backward_dk.bin", sh)) < 1e-4
    assert _rel(dv, load("flash_attn2", "expected_backward_dv.bin", sh)) < 1e-4


def test_attention_bwd_oracle_causal_gqa_vs_torch():
    torch = pytest.importorskip("torch")
    r = np.random.default_rng(3)
    B, Hq, Hkv, Sq, Sk, D = 2, 4, 2, 9, 13, 16
    q = r.standard_normal((B, Hq, Sq, D)).astype(np.float32)
    k = r.standard_normal((B, Hkv, Sk, D)).astype(np.float32)
    v = r.standard_normal((B, Hkv, Sk, D)).astype(np.float32)
    do = r.standard_normal((B, Hq, Sq, D)).astype(np.float32)
    o, lse = oracle.attention(q, k, v, 0.25, True)
    dq, dk, dv = oracle.attention_bwd(q, k, v, o, do, lse, 0.25, True)
    tq, tk, tv = (torch.from_numpy(a).double().requires_grad_(True) for a in (q, k, v))
    kk, vv = tk.repeat_interleave(Hq // Hkv, 1), tv.repeat_interleave(Hq // Hkv, 1)
    s = tq @ kk.transpose(-1, -2) * 0.25
    mask = torch.ones(Sq, Sk, dtype=torch.bool).tril(Sk - Sq)
    s = s.masked_fill(~mask, float("-inf"))
    (torch.softmax(s, -1) @ vv).backward(torch.from_numpy(do).double())
    assert _rel(dq, tq.grad.numpy()) < 1e-5
    assert _rel(dk, tk.grad.numpy()) < 1e-5
    assert _rel(dv, tv.grad.numpy()) < 1e-5


def test_linear_bwd_oracle_golden():
    x = load("linear", "input.bin", (64, 64))
    w = load("linear", "weight.bin", (48, 64))
    dy = load("linear", "dy.bin", (64, 48))
    dx, dw, db = oracle.linear_bwd(x, w, dy)
    assert _rel(dx, load("linear", "expected_dx.bin", (64, 64))) < 1e-5
    assert _rel(dw, load("linear", "expected_dw.bin", (48, 64))) < 1e-5
    assert _rel(db, load("linear", "expected_db.bin", (48,))) < 1e-5


@pytest.mark.parametrize("name,pad,oh", [("conv2d", 0, 6), ("conv2d_padded", 1, 8)])
def test_conv2d_bwd_oracle_golden(name, pad, oh):
    x = load(name, "x.bin", (1, 2, 8, 8))
    w = load(name, "w.bin", (4, 2, 3, 3))
    dy = load(name, "dy.bin", (1, 4, oh, oh))
    dx, dw = oracle.conv2d_bwd(dy, x, w, 1, pad)
    assert _rel(dx, load(name, "expected_dx.bin", (1, 2, 8, 8))) < 1e-5
    assert _rel(dw, load(name, "expected_dw.bin", (4, 2, 3, 3))) < 1e-5


def test_conv2d_bwd_oracle_strided_vs_torch():
    torch = pytest.importorskip("torch")
    r = np.random.default_rng(4)
    x = r.standard_normal((2, 3, 11, 9)).astype(np.float32)
    w = r.standard_normal((5, 3, 3, 3)).astype(np.float32)
    tx, tw = torch.from_numpy(x).double().requires_grad_(True), torch.from_numpy(w).double().requires_grad_(True)
    y = torch.nn.functional.conv2d(tx, tw, stride=2, padding=1)
    dy = r.standard_normal(tuple(y.shape)).astype(np.float32)
    y.backward(torch.from_numpy(dy).double())
    dx, dw = oracle.conv2d_bwd(dy, x, w, 2, 1)
    assert _rel(dx, tx.grad.numpy()) < 1e-5
    assert _rel(dw, tw.grad.numpy()) < 1e-5


def test_rmsnorm_bwd_oracle_vs_torch():
    # the reference holds no rmsnorm backward vectors; torch autograd of the
    # forward formula (rmsnorm.rs:40-122) is the cross-check
    torch = pytest.importorskip("torch")
    r = np.random.default_rng(5)
    x = r.uniform(-2, 2, (16, 128)).astype(np.float32)
    w = r.uniform(0.5, 1.5, 128).astype(np.float32)
    dy = r.uniform(-1, 1, (16, 128)).astype(np.float32)
    _, rrms = oracle.rmsnorm(x, w, 1e-8)
    dw0 = r.standard_normal(128).astype(np.float32)
    dx, dw = oracle.rmsnorm_bwd(dy, x, w, rrms, dw0)
    tx, tw = torch.from_numpy(x).double().requires_grad_(True), torch.from_numpy(w).double().requires_grad_(True)
    y = tx * torch.rsqrt((tx * tx).mean(-1, keepdim=True) + 1e-8) * tw
    y.backward(torch.from_numpy(dy).double())
    assert _rel(dx, tx.grad.numpy()) < 1e-5
    assert _rel(dw - dw0, tw.grad.numpy()) < 1e-5


def test_rmsnorm_bwd_oracle_matches_reference_formula_at_unit_gain():
    # with w == 1 the reference's dx line (rmsnorm.rs:232) and the gradient agree
    r = np.random.default_rng(6)
    x = r.uniform(-2, 2, (8, 64)).astype(np.float32)
    dy = r.uniform(-1, 1, (8, 64)).astype(np.float32)
    w = np.ones(64, np.float32)
    _, rrms = oracle.rmsnorm(x, w, 1e-8)
    dx, _ = oracle.rmsnorm_bwd(dy, x, w, rrms)
    rr = rrms.astype(np.float64)[:, None]
    dot = (dy.astype(np.float64) * w * x).sum(-1, keepdims=True)
    ref = rr * w * (dy - x * rr * rr * dot / 64)
    assert _rel(dx, ref) < 1e-6
