"""GPU parity of conv2d (+ bias, folded BN, activation), BN folding and
batch-norm inference against the reference fixtures and the CPU oracle."""
import numpy as np
import pytest

from gpu_util import BF16_TOL, F32_TOL, assert_close, bf16_round, dev, no_device_error, np_of, rng, to_gpu, torch
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


@pytest.mark.parametrize("name,pad,oh", [("conv2d", 0, 6), ("conv2d_padded", 1, 8)])
def test_conv2d_golden_f32(name, pad, oh):
    x = load(name, "x.bin", (1, 2, 8, 8))
    w = load(name, "w.bin", (4, 2, 3, 3))
    y = ops().conv2d(to_gpu(x), to_gpu(w), pad=pad)
    assert_close(np_of(y), load(name, "expected_forward.bin", (1, 4, oh, oh)), F32_TOL)


def test_batchnorm_golden_and_fold():
    x = load("batchnorm", "x.bin", (64, 32))
    args = [to_gpu(load("batchnorm", f)) for f in ("weight.bin", "bias.bin", "running_mean.bin", "running_var.bin")]
    y = ops().batch_norm_inference(to_gpu(x), *args, eps=1e-5)
    assert_close(np_of(y), load("batchnorm", "expected_forward_inference.bin", (64, 32)), F32_TOL)
    r = rng(1)
    g, be, mu, var, b = (r.uniform(0.5, 1.5, 64), r.normal(0, .1, 64), r.normal(0, .1, 64), r.uniform(.5, 1.5, 64),
                         r.normal(0, .1, 64))
    sc, sh = ops().bn_fold(*(to_gpu(a) for a in (g, be, mu, var)), eps=1e-5, bias=to_gpu(b))
    rsc, rsh = oracle.bn_fold(g, be, mu, var, 1e-5, b)
    assert_close(np_of(sc), rsc, 1e-6)
    assert_close(np_of(sh), rsh, 1e-6)


def _conv_case(B, C, Co, H, W, k, stride, pad, act, dtype, seed, with_bn=True):
    r = rng(seed)
    x = r.standard_normal((B, C, H, W)).astype(np.float32)
    w = (r.standard_normal((Co, C, k, k)) * np.sqrt(2.0 / (C * k * k))).astype(np.float32)
    bias = r.normal(0, 0.1, Co).astype(np.float32)
    if dtype == torch.bfloat16:
        x, w = bf16_round(x), bf16_round(w)
    sc = sh = None
    if with_bn:
        sc, sh = oracle.bn_fold(r.uniform(0.5, 1.5, Co), r.normal(0, .1, Co), r.normal(0, .1, Co),
                                r.uniform(0.5, 1.5, Co), 1e-5, bias)
    ref = oracle.conv2d(x, w, bias=bias, scale=sc, shift=sh, stride=stride, pad=pad, act=act)
    y = ops().conv2d(to_gpu(x, dtype), to_gpu(w, dtype), bias=to_gpu(bias),
                     scale=None if sc is None else to_gpu(sc), shift=None if sh is None else to_gpu(sh),
                     stride=stride, pad=pad, act=act)
    return np_of(y), ref


@pytest.mark.parametrize("B,C,Co,H,W,k,p,act", [(2, 64, 64, 24, 24, 3, 1, "relu"), (1, 3, 40, 20, 16, 3, 1, "silu"),
                                                (2, 128, 96, 16, 32, 3, 1, None), (32, 64, 64, 56, 56, 3, 1, "relu"),
                                                (2, 32, 64, 16, 16, 1, 0, "relu"), (1, 16, 32, 20, 24, 5, 2, None),
                                                (1, 8, 64, 22, 24, 7, 3, "relu"), (1, 24, 72, 30, 42, 3, 0, None),
                                                (1, 16, 64, 10, 80, 3, 1, "relu")])   # two 64-column prep tiles
def test_conv2d_bf16_tensor_cores(B, C, Co, H, W, k, p, act):
    got, ref = _conv_case(B, C, Co, H, W, k, 1, p, act, torch.bfloat16, seed=B + C + Co + k)
    assert_close(got, ref, BF16_TOL)


def test_conv2d_pack_weights_exact():
    r = rng(11)
    w = bf16_round(r.standard_normal((72, 24, 3, 5)))
    got = np_of(ops().conv2d_pack_weights(to_gpu(w, torch.bfloat16)))
    np.testing.assert_array_equal(got, w.transpose(0, 2, 3, 1))


@pytest.mark.parametrize("B,C,H,W,layers,act", [(32, 64, 56, 56, 4, "relu"), (3, 64, 20, 24, 3, "silu"),
                                                 (2, 32, 17, 16, 2, None)])
def test_conv2d_nhwc_chain(B, C, H, W, layers, act):
    """The C2 stage as an executor runs it: NCHW in, NHWC between the convolutions,
    NCHW out, weights packed once; against the oracle's NCHW chain (each layer's
    input rounded to bf16, as the device stores it), and the NHWC intermediate
    against the oracle's first layer."""
    r = rng(B + C + layers)
    x = bf16_round(r.standard_normal((B, C, H, W)))
    params = []
    for _ in range(layers):
        w = bf16_round(r.standard_normal((C, C, 3, 3)) * np.sqrt(2.0 / (C * 9)))
        bias = r.normal(0, 0.1, C).astype(np.float32)
        sc, sh = oracle.bn_fold(r.uniform(0.5, 1.5, C), r.normal(0, .1, C), r.normal(0, .1, C),
                                r.uniform(0.5, 1.5, C), 1e-5, bias)
        params.append((w, sc, sh))
    ref, refs = x, []
    for w, sc, sh in params:
        ref = bf16_round(oracle.conv2d(ref, w, scale=sc, shift=sh, pad=1, act=act))
        refs.append(ref)
    y = to_gpu(x, torch.bfloat16)
    outs = []
    for i, (w, sc, sh) in enumerate(params):
        wp = ops().conv2d_pack_weights(to_gpu(w, torch.bfloat16))
        y = ops().conv2d(y, wp, scale=to_gpu(sc), shift=to_gpu(sh), pad=1, act=act, x_nhwc=i > 0,
                         y_nhwc=i < layers - 1, w_packed=True)
        outs.append(y)
    assert tuple(outs[0].shape) == (B, H, W, C)
    assert_close(np_of(outs[0]).transpose(0, 3, 1, 2), refs[0], BF16_TOL, "NHWC intermediate")
    assert tuple(y.shape) == (B, C, H, W)
    assert_close(np_of(y), refs[-1], BF16_TOL, "stage output")


@pytest.mark.parametrize("Cin,Cout,H,W", [(16, 24, 18, 16), (64, 72, 20, 24), (64, 48, 9, 8), (32, 16, 33, 40)])
def test_conv2d_nhwc_out_channels(Cin, Cout, H, W):
    """NHWC output written from registers: 16-byte stores (Cout % 16 == 8), 32-byte
    stores (Cout % 16 == 0), a partial second channel block (Cout 72), clipped rows."""
    r = rng(Cin + Cout + H)
    x = bf16_round(r.standard_normal((2, Cin, H, W)))
    w = bf16_round(r.standard_normal((Cout, Cin, 3, 3)) * np.sqrt(2.0 / (Cin * 9)))
    sc = r.uniform(0.5, 1.5, Cout).astype(np.float32)
    sh = r.normal(0, 0.1, Cout).astype(np.float32)
    ref = bf16_round(oracle.conv2d(x, w, scale=sc, shift=sh, pad=1, act="relu"))
    y = ops().conv2d(to_gpu(x, torch.bfloat16), to_gpu(w, torch.bfloat16), scale=to_gpu(sc), shift=to_gpu(sh), pad=1,
                     act="relu", y_nhwc=True)
    assert tuple(y.shape) == (2, H, W, Cout)
    assert_close(np_of(y).transpose(0, 3, 1, 2), ref, BF16_TOL, "NHWC output")


def test_conv2d_layout_flags_rejected():
    from teenygrad_b200._lib import TB_ERR_UNSUPPORTED, TeenyError
    r = rng(3)
    x = to_gpu(bf16_round(r.standard_normal((1, 12, 16, 16))), torch.bfloat16)     # Cin % 8 != 0
    w = to_gpu(bf16_round(r.standard_normal((16, 12, 3, 3))), torch.bfloat16)
    with pytest.raises(TeenyError) as e:
        ops().conv2d(x.permute(0, 2, 3, 1).contiguous(), w, pad=1, x_nhwc=True)
    assert e.value.status == TB_ERR_UNSUPPORTED
    xf = to_gpu(r.standard_normal((1, 16, 16, 16)).astype(np.float32))           # f32: CUDA-core path only
    wf = to_gpu(r.standard_normal((16, 16, 3, 3)).astype(np.float32))
    with pytest.raises(TeenyError) as e:
        ops().conv2d(xf, wf, pad=1, y_nhwc=True)
    assert e.value.status == TB_ERR_UNSUPPORTED
    x7 = to_gpu(bf16_round(r.standard_normal((1, 16, 20, 24))), torch.bfloat16)   # 7 x 7: conv_tc_kernel
    w7 = to_gpu(bf16_round(r.standard_normal((64, 16, 7, 7))), torch.bfloat16)
    with pytest.raises(TeenyError) as e:
        ops().conv2d(x7, w7, pad=3, y_nhwc=True)
    assert e.value.status == TB_ERR_UNSUPPORTED
    no_device_error()


def test_conv2d_bf16_cuda_core_shapes():
    got, ref = _conv_case(2, 16, 24, 17, 19, 3, 2, 1, "relu", torch.bfloat16, seed=5)   # stride 2, OW % 8 != 0
    assert_close(got, ref, BF16_TOL)


@pytest.mark.parametrize("B,C,Co,H,W,k,s,p", [(1, 64, 64, 56, 56, 3, 1, 1), (2, 5, 7, 9, 11, 3, 2, 0), (1, 8, 16, 10, 10, 1, 1, 0)])
def test_conv2d_f32(B, C, Co, H, W, k, s, p):
    got, ref = _conv_case(B, C, Co, H, W, k, s, p, "relu", torch.float32, seed=k + s + C)
    assert_close(got, ref, F32_TOL)


@pytest.mark.parametrize("B,C,Co,H,W,act,bn", [(2, 16, 128, 9, 16, "silu", True), (3, 8, 64, 5, 8, None, False),
                                                (1, 64, 64, 3, 128, "relu", True), (2, 24, 64, 7, 40, "relu", False)])
def test_conv2d_f32_direct3x3(B, C, Co, H, W, act, bn):
    """The fp32 3 x 3 / stride 1 / pad 1 direct kernel: two output-channel blocks,
    the narrowest and widest rows it takes, bias without BN, SiLU."""
    got, ref = _conv_case(B, C, Co, H, W, 3, 1, 1, act, torch.float32, seed=H + W + C, with_bn=bn)
    assert_close(got, ref, F32_TOL)
    no_device_error()


def test_conv2d_plain_bias_no_bn():
    got, ref = _conv_case(1, 64, 64, 16, 16, 3, 1, 1, None, torch.bfloat16, seed=11, with_bn=False)
    assert_close(got, ref, BF16_TOL)
