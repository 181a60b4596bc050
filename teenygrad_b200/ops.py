"""Host-side operator surface over the C ABI, on torch CUDA tensors.

The reference dispatches each graph node to a kernel struct implementing
``RuntimeOp`` (core/teeny-core/src/model/mod.rs:78-330): ``pack_args`` +
``grid`` + a launch.  Here each op is a function (and a class with the
reference kernel's name, for code written against that surface) that checks
shapes, allocates the output and calls the matching ``tb_*`` entry point on
the current torch stream.  Errors surface as :class:`TeenyError` (the
reference returns ``anyhow::Result``).

torch is used only for device memory and streams.
"""
from __future__ import annotations

import ctypes
import math

import torch

from ._lib import (TB_ACT, TB_BF16, TB_EPI_BIAS, TB_EPI_OUT_F32, TB_EPI_RESIDUAL, TB_EPI_SWIGLU,
                   TB_F32, TeenyError, check, lib)

_DT = {torch.float32: TB_F32, torch.bfloat16: TB_BF16}
_ctxs: dict[int, ctypes.c_void_p] = {}


def context(device: int | None = None) -> ctypes.c_void_p:
    """Per-device tb_ctx, bound to torch's current stream at each call."""
    if device is None:
        device = torch.cuda.current_device()
    ctx = _ctxs.get(device)
    if ctx is None:
        ctx = ctypes.c_void_p()
        st = lib().tb_init(ctypes.byref(ctx), ctypes.c_int(device))
        if st != 0:
            raise TeenyError(st, f"tb_init(device={device}) failed: needs an sm_100 GPU")
        _ctxs[device] = ctx
    lib().tb_set_stream(ctx, ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream))
    return ctx


def device_error(clear: bool = True) -> int:
    ctx = context()
    code = ctypes.c_int(0)
    check(ctx, lib().tb_device_error(ctx, ctypes.byref(code), ctypes.c_int(int(clear))))
    return code.value


def _p(t):
    return ctypes.c_void_p(0 if t is None else t.data_ptr())


def _dt(t):
    if t.dtype not in _DT:
        raise TeenyError(5, f"unsupported dtype {t.dtype}")
    return _DT[t.dtype]


def _cuda(*ts):
    for t in ts:
        if t is not None:
            if not t.is_cuda:
                raise TeenyError(1, "tensors must be on a CUDA device (no CPU fallback)")
            if not t.is_contiguous():
                raise TeenyError(2, "tensors must be contiguous")


_i64 = ctypes.c_int64
_f = ctypes.c_float


# --------------------------------------------------------------- norms ----
def rms_norm(x, w, eps=1e-8, return_rrms=False):
    """rms_norm_forward (nn/norm/rmsnorm.rs:40-122); x [..., N]."""
    _cuda(x, w)
    N = x.shape[-1]
    M = x.numel() // N
    y = torch.empty_like(x)
    rrms = torch.empty(M, device=x.device, dtype=torch.float32) if return_rrms else None
    ctx = context()
    check(ctx, lib().tb_rmsnorm_fwd(ctx, _dt(x), _p(x), _p(w), _p(y), _p(rrms), _i64(M), _i64(N), _f(eps)))
    return (y, rrms) if return_rrms else y


def layer_norm(x, w, b, eps=1e-5):
    """layer_norm_forward_inference (nn/norm/layernorm.rs:43-157)."""
    _cuda(x, w, b)
    N = x.shape[-1]
    y = torch.empty_like(x)
    ctx = context()
    check(ctx, lib().tb_layernorm_fwd(ctx, _dt(x), _p(x), _p(w), _p(b), _p(y), _i64(x.numel() // N), _i64(N), _f(eps)))
    return y


# --------------------------------------------------------- elementwise ----
def activation(kind, x):
    _cuda(x)
    y = torch.empty_like(x)
    ctx = context()
    check(ctx, lib().tb_act_fwd(ctx, ctypes.c_int(TB_ACT[kind]), _dt(x), _p(x), _p(y), _i64(x.numel())))
    return y


def silu(x):
    return activation("silu", x)


def gelu_tanh(x):
    return activation("gelu_tanh", x)


def relu(x):
    return activation("relu", x)


def sigmoid(x):
    return activation("sigmoid", x)


def swiglu(gate, up):
    _cuda(gate, up)
    y = torch.empty_like(gate)
    ctx = context()
    check(ctx, lib().tb_swiglu_fwd(ctx, _dt(gate), _p(gate), _p(up), _p(y), _i64(gate.numel())))
    return y


def add(a, b):
    _cuda(a, b)
    y = torch.empty_like(a)
    ctx = context()
    check(ctx, lib().tb_add_fwd(ctx, _dt(a), _p(a), _p(b), _p(y), _i64(a.numel())))
    return y


# --------------------------------------------------------------- linear ---
def linear(x, w, bias=None, residual=None, swiglu=False, out_f32=False):
    """linear_forward (nn/mlp/linear.rs:22-117): y = x w^T (+ bias) (+ residual).

    swiglu=True expects w rows interleaved in blocks of 128 (gate, up) and
    returns silu(gate) * up with N/2 columns (see interleave_gate_up)."""
    _cuda(x, w, bias, residual)
    K = x.shape[-1]
    M = x.numel() // K
    N = w.shape[0]
    flags = (TB_EPI_BIAS if bias is not None else 0) | (TB_EPI_RESIDUAL if residual is not None else 0)
    flags |= (TB_EPI_SWIGLU if swiglu else 0) | (TB_EPI_OUT_F32 if out_f32 else 0)
    ncol = N // 2 if swiglu else N
    y = torch.empty(*x.shape[:-1], ncol, device=x.device, dtype=torch.float32 if out_f32 else x.dtype)
    if bias is not None and bias.dtype != torch.float32:
        bias = bias.float().contiguous()
    ctx = context()
    check(ctx, lib().tb_linear_fwd(ctx, _dt(x), _p(x), _p(w), _p(bias), _p(residual), _p(y),
                                   _i64(M), _i64(N), _i64(K), ctypes.c_int(flags)))
    return y


class _LinearStep(ctypes.Structure):
    _fields_ = [("x", ctypes.c_void_p), ("ldx", ctypes.c_int64), ("w", ctypes.c_void_p),
                ("norm_w", ctypes.c_void_p), ("norm_eps", ctypes.c_float), ("residual", ctypes.c_void_p),
                ("y", ctypes.c_void_p), ("ldy", ctypes.c_int64), ("N", ctypes.c_int64), ("K", ctypes.c_int64),
                ("flags", ctypes.c_int)]


def linear_chain(steps):
    """Dependent decode linear layers in one persistent launch (tb_linear_chain_fwd).

    steps: dicts with x [M, K] and w [N, K] (bf16), y (the output tensor, written;
    step i + 1 may take step i's y as its x or residual) and optional norm_w
    ([K] RMSNorm gains fused in front of the matmul), eps, residual (may be y),
    swiglu.  Every step has the same M <= 64 rows."""
    arr = (_LinearStep * len(steps))()
    M = None
    for i, st in enumerate(steps):
        x, w, y = st["x"], st["w"], st["y"]
        _cuda(x, w, y, st.get("norm_w"), st.get("residual"))
        K = x.shape[-1]
        m = x.numel() // K
        M = m if M is None else M
        if m != M:
            raise ValueError("linear_chain: every step needs the same number of rows")
        flags = (TB_EPI_SWIGLU if st.get("swiglu") else 0) | (TB_EPI_RESIDUAL if st.get("residual") is not None else 0)
        addr = lambda t: None if t is None else t.data_ptr()  # noqa: E731
        arr[i] = _LinearStep(addr(x), x.stride(-2) if x.dim() > 1 else K, addr(w), addr(st.get("norm_w")),
                             float(st.get("eps", 1e-5)), addr(st.get("residual")), addr(y),
                             y.stride(-2) if y.dim() > 1 else y.shape[-1], w.shape[0], K, flags)
    ctx = context()
    check(ctx, lib().tb_linear_chain_fwd(ctx, arr, ctypes.c_int(len(steps)), _i64(M)))


TB_OP = {"linear": 0, "matmul": 1, "int8_linear": 2, "rmsnorm": 3, "layernorm": 4, "act": 5, "attn": 6,
         "conv2d": 7, "quantize_int8": 8}


def output_row_stride(op, dtype, row_elems):
    """RuntimeOp::forward_output_row_stride (core/teeny-core/src/model/mod.rs:100):
    the row stride an executor allocates for the op's output rows."""
    out = ctypes.c_int64(0)
    dt = _DT[dtype] if isinstance(dtype, torch.dtype) else dtype
    check(None, lib().tb_output_row_stride(ctypes.c_int(TB_OP[op]), ctypes.c_int(dt), _i64(row_elems), ctypes.byref(out)))
    return out.value


def linear_padded(x, w, bias=None):
    """LinearForward as the reference executor runs it (nn/mlp/linear.rs:251-300):
    the output buffer's rows are padded to 16 bytes (output_row_stride) and the
    kernel writes the first N columns of each.  Returns (buffer [M, stride], y view [M, N])."""
    _cuda(x, w, bias)
    K = x.shape[-1]
    M = x.numel() // K
    N = w.shape[0]
    ld = output_row_stride("linear", x.dtype, N)
    buf = torch.full((M, ld), float("nan"), device=x.device, dtype=x.dtype)
    if bias is not None and bias.dtype != torch.float32:
        bias = bias.float().contiguous()
    ctx = context()
    check(ctx, lib().tb_linear_fwd_strided(ctx, _dt(x), _p(x), _i64(K), _p(w), _p(bias), _p(None), _p(buf), _i64(ld),
                                           _i64(M), _i64(N), _i64(K),
                                           ctypes.c_int(TB_EPI_BIAS if bias is not None else 0)))
    return buf, buf[:, :N]


def interleave_gate_up(w_gate, w_up, block=128):
    """[F, K] gate and up weights -> [2F, K] in the (gate block, up block) order
    the fused SwiGLU epilogue expects."""
    F, K = w_gate.shape
    g = w_gate.reshape(F // block, block, K)
    u = w_up.reshape(F // block, block, K)
    return torch.stack([g, u], dim=1).reshape(2 * F, K).contiguous()


def matmul(a, b):
    """matmul_forward (math/gemm.rs:44-105): c = a @ b, b [K, N]."""
    _cuda(a, b)
    M, K = a.shape
    N = b.shape[1]
    c = torch.empty(M, N, device=a.device, dtype=a.dtype)
    ctx = context()
    check(ctx, lib().tb_matmul_fwd(ctx, _dt(a), _p(a), _p(b), _p(c), _i64(M), _i64(N), _i64(K)))
    return c


# ----------------------------------------------------------------- int8 ---
def quantize_int8(w):
    """quantize_affine, symmetric per output channel (teeny-quant affine.rs:55-148)."""
    _cuda(w)
    N, K = w.shape
    q = torch.empty(N, K, device=w.device, dtype=torch.int8)
    s = torch.empty(N, device=w.device, dtype=torch.float32)
    ctx = context()
    fn = lib().tb_quantize_int8 if w.dtype == torch.float32 else lib().tb_quantize_int8_bf16
    check(ctx, fn(ctx, _p(w), _p(q), _p(s), _i64(N), _i64(K)))
    return q, s


def dequantize_int8(q, s):
    _cuda(q, s)
    N, K = q.shape
    w = torch.empty(N, K, device=q.device, dtype=torch.float32)
    ctx = context()
    check(ctx, lib().tb_dequantize_int8(ctx, _p(q), _p(s), _p(w), _i64(N), _i64(K)))
    return w


def int8_linear(x, q, s, residual=None, swiglu=False, out_f32=False):
    _cuda(x, q, s, residual)
    K = x.shape[-1]
    M = x.numel() // K
    N = q.shape[0]
    flags = (TB_EPI_RESIDUAL if residual is not None else 0) | (TB_EPI_SWIGLU if swiglu else 0)
    flags |= TB_EPI_OUT_F32 if out_f32 else 0
    ncol = N // 2 if swiglu else N
    y = torch.empty(*x.shape[:-1], ncol, device=x.device, dtype=torch.float32 if out_f32 else x.dtype)
    ctx = context()
    check(ctx, lib().tb_int8_linear_fwd(ctx, _p(x), _p(q), _p(s), _p(residual), _p(y), _i64(M), _i64(N),
                                        _i64(K), ctypes.c_int(flags)))
    return y


# ------------------------------------------------------------ attention ---
def attention(q, k, v, scale=None, causal=False, return_lse=False):
    """flash_attention2_forward (nn/attention/flash_attn2.rs:53-158) + causal + GQA.
    q [B, Hq, Sq, D], k/v [B, Hkv, Sk, D]."""
    _cuda(q, k, v)
    B, Hq, Sq, D = q.shape
    Hkv, Sk = k.shape[1], k.shape[2]
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    o = torch.empty_like(q)
    lse = torch.empty(B, Hq, Sq, device=q.device, dtype=torch.float32) if return_lse else None
    ctx = context()
    check(ctx, lib().tb_attn_fwd(ctx, _dt(q), _p(q), _p(k), _p(v), _p(o), _p(lse), ctypes.c_int(B),
                                 ctypes.c_int(Hq), ctypes.c_int(Hkv), ctypes.c_int(Sq), ctypes.c_int(Sk),
                                 ctypes.c_int(D), _f(scale), ctypes.c_int(int(causal))))
    return (o, lse) if return_lse else o


# --------------------------------------------------------- decoder ops ----
def rope(x, pos, theta=10000.0):
    """x [T, H, D], pos [T] int32."""
    _cuda(x, pos)
    T, H, D = x.shape
    y = torch.empty_like(x)
    ctx = context()
    check(ctx, lib().tb_rope_fwd(ctx, _dt(x), _p(x), _p(pos), _p(y), _i64(T), ctypes.c_int(H), ctypes.c_int(D), _f(theta)))
    return y


def embedding(table, ids):
    _cuda(table, ids)
    T = ids.numel()
    D = table.shape[1]
    y = torch.empty(T, D, device=table.device, dtype=table.dtype)
    ctx = context()
    check(ctx, lib().tb_embedding_fwd(ctx, _dt(table), _p(table), _p(ids), _p(y), _i64(T), _i64(D), _i64(table.shape[0])))
    return y


def argmax(x):
    _cuda(x)
    M, N = x.shape
    out = torch.empty(M, device=x.device, dtype=torch.int32)
    ctx = context()
    check(ctx, lib().tb_argmax_fwd(ctx, _dt(x), _p(x), _p(out), _i64(M), _i64(N)))
    return out


# ------------------------------------------- reference kernel-struct names --
class _Op:
    fn = None

    def __init__(self, **consts):
        self.consts = consts

    def __call__(self, *args, **kw):
        return type(self).fn(*args, **{**self.consts, **kw})


class RmsNormForward(_Op):
    fn = staticmethod(rms_norm)


class LayerNormForwardInference(_Op):
    fn = staticmethod(layer_norm)


class SiluForward(_Op):
    fn = staticmethod(silu)


class GeluForward(_Op):
    fn = staticmethod(gelu_tanh)


class ReluForward(_Op):
    fn = staticmethod(relu)


class LinearForward(_Op):
    fn = staticmethod(linear)


class MatMulForward(_Op):
    fn = staticmethod(matmul)


class FlashAttention2Forward(_Op):
    fn = staticmethod(attention)


# ----------------------------------------------------------------- conv ---
def bn_fold(gamma, beta, mean, var, eps=1e-5, bias=None):
    """BN folding of nn/fused/conv2d_bn_silu.rs:33-35 (f32 [C])."""
    _cuda(gamma, beta, mean, var, bias)
    C = gamma.numel()
    scale = torch.empty(C, device=gamma.device, dtype=torch.float32)
    shift = torch.empty_like(scale)
    ctx = context()
    check(ctx, lib().tb_bn_fold(ctx, _p(gamma), _p(beta), _p(mean), _p(var), _p(bias), _f(eps), _p(scale), _p(shift),
                                ctypes.c_int(C)))
    return scale, shift


def batch_norm_inference(x, gamma, beta, mean, var, eps=1e-5):
    """batch_norm_2d_nchw_forward_inference (nn/norm/batchnorm.rs:574-686); x [B, C, ...]."""
    _cuda(x, gamma, beta, mean, var)
    B, C = x.shape[0], x.shape[1]
    HW = x.numel() // max(1, B * C)
    y = torch.empty_like(x)
    ctx = context()
    check(ctx, lib().tb_batchnorm_fwd(ctx, _dt(x), _p(x), _p(gamma), _p(beta), _p(mean), _p(var), _p(y), _i64(B),
                                      _i64(C), _i64(HW), _f(eps)))
    return y


_CONV_ACT = {None: -1, "relu": 2, "silu": 0}


def conv2d(x, w, bias=None, scale=None, shift=None, stride=1, pad=0, act=None, x_nhwc=False, y_nhwc=False,
           w_packed=False):
    """conv2d_bias_forward (nn/conv/conv2d.rs:643-764) + folded-BN epilogue
    (nn/fused/conv2d_bn_silu.rs:141-170); NCHW, groups = 1.

    Layout options for chained convolutions (tb_conv2d_fwd_ex, bf16 tensor-core
    shapes): x_nhwc takes x as [B, H, W, C], y_nhwc returns y as [B, OH, OW, Co],
    w_packed takes w as [Co, KH, KW, C] (conv2d_pack_weights)."""
    _cuda(x, w, bias, scale, shift)
    if x_nhwc:
        B, H, W, C = x.shape
    else:
        B, C, H, W = x.shape
    if w_packed:
        Co, KH, KW, _ = w.shape
    else:
        Co, _, KH, KW = w.shape
    OH = (H + 2 * pad - KH) // stride + 1
    OW = (W + 2 * pad - KW) // stride + 1
    shape = (B, OH, OW, Co) if y_nhwc else (B, Co, OH, OW)
    y = torch.empty(*shape, device=x.device, dtype=x.dtype)
    flags = (1 if x_nhwc else 0) | (2 if y_nhwc else 0) | (4 if w_packed else 0)
    nbytes = ctypes.c_size_t(0)
    if not (x_nhwc and w_packed):
        st = lib().tb_conv2d_workspace_size(ctypes.c_int(_dt(x)),
                                            *(ctypes.c_int(v) for v in (B, C, Co, H, W, KH, KW, stride, pad)),
                                            ctypes.byref(nbytes))
        check(None, st)
    ws = torch.empty(max(1, nbytes.value), device=x.device, dtype=torch.uint8) if nbytes.value else None
    ctx = context()
    f = [t if t is None or t.dtype == torch.float32 else t.float().contiguous() for t in (bias, scale, shift)]
    check(ctx, lib().tb_conv2d_fwd_ex(ctx, ctypes.c_int(_dt(x)), _p(x), _p(w), _p(f[0]), _p(f[1]), _p(f[2]), _p(y),
                                      *(ctypes.c_int(v) for v in (B, C, Co, H, W, KH, KW, stride, pad, _CONV_ACT[act],
                                                                   flags)),
                                      _p(ws), ctypes.c_size_t(nbytes.value)))
    return y


def conv2d_pack_weights(w):
    """w [Co, C, KH, KW] bf16 -> [Co, KH, KW, C], the layout conv2d(w_packed=True) takes."""
    _cuda(w)
    Co, C, KH, KW = w.shape
    out = torch.empty(Co, KH, KW, C, device=w.device, dtype=w.dtype)
    ctx = context()
    check(ctx, lib().tb_conv2d_pack_weights(ctx, ctypes.c_int(_dt(w)), _p(w), _p(out),
                                            *(ctypes.c_int(v) for v in (Co, C, KH, KW))))
    return out


class Conv2dBiasForward(_Op):
    fn = staticmethod(conv2d)


# --------------------------------------------------------------- backward ---
def _workspace(op, dtype, shape, device):
    n = ctypes.c_size_t(0)
    arr = (ctypes.c_int64 * len(shape))(*shape)
    check(None, lib().tb_workspace_bytes(ctypes.c_int(TB_OP[op]), ctypes.c_int(dtype), arr, ctypes.c_int(len(shape)),
                                         ctypes.byref(n)))
    return torch.empty(max(n.value, 16), dtype=torch.uint8, device=device), n.value


TB_OP.update({"rmsnorm_bwd": 9, "linear_bwd": 10, "attn_bwd": 11, "conv2d_bwd": 12})


def rms_norm_backward(dy, x, w, rrms, dw=None):
    """rms_norm_backward (nn/norm/rmsnorm.rs:125-277): returns (dx, dw); dw (f32 [N])
    accumulates into the given tensor (zeros when None)."""
    _cuda(dy, x, w, rrms, dw)
    N = x.shape[-1]
    M = x.numel() // N
    dx = torch.empty_like(x)
    if dw is None:
        dw = torch.zeros(N, device=x.device, dtype=torch.float32)
    ws, nb = _workspace("rmsnorm_bwd", _dt(x), (M, N), x.device)
    ctx = context()
    check(ctx, lib().tb_rmsnorm_bwd(ctx, _dt(x), _p(dy), _p(x), _p(w), _p(rrms), _p(dx), _p(dw), _i64(M), _i64(N),
                                    _p(ws), ctypes.c_size_t(nb)))
    return dx, dw


def linear_backward(x, w, dy, bias=True):
    """linear_backward (nn/mlp/linear.rs:119-249): (dx, dw, db) of y = x w^T + b."""
    _cuda(x, w, dy)
    K = x.shape[-1]
    M = x.numel() // K
    N = w.shape[0]
    dx = torch.empty_like(x)
    dw = torch.empty_like(w)
    db = torch.empty(N, device=x.device, dtype=torch.float32) if bias else None
    ws, nb = _workspace("linear_bwd", _dt(x), (M, N, K), x.device)
    ctx = context()
    check(ctx, lib().tb_linear_bwd(ctx, _dt(x), _p(x), _p(w), _p(dy), _p(dx), _p(dw), _p(db), _i64(M), _i64(N),
                                   _i64(K), _p(ws), ctypes.c_size_t(nb)))
    return dx, dw, db


def attention_backward(q, k, v, o, do, lse, scale=None, causal=False):
    """flash_attention2_backward_dq / _dkv (nn/attention/flash_attn2.rs:160-447)
    with causal masking and GQA: returns (dq, dk, dv)."""
    _cuda(q, k, v, o, do, lse)
    B, Hq, Sq, D = q.shape
    Hkv, Sk = k.shape[1], k.shape[2]
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    ws, nb = _workspace("attn_bwd", _dt(q), (B, Hq, Sq), q.device)
    ctx = context()
    check(ctx, lib().tb_attn_bwd(ctx, _dt(q), _p(q), _p(k), _p(v), _p(o), _p(do), _p(lse), _p(dq), _p(dk), _p(dv),
                                 ctypes.c_int(B), ctypes.c_int(Hq), ctypes.c_int(Hkv), ctypes.c_int(Sq), ctypes.c_int(Sk),
                                 ctypes.c_int(D), _f(scale), ctypes.c_int(int(causal)), _p(ws), ctypes.c_size_t(nb)))
    return dq, dk, dv


def conv2d_backward(dy, x, w, stride=1, pad=0):
    """conv2d_backward (nn/conv/conv2d.rs:395-521), groups = 1: returns (dx, dw)."""
    _cuda(dy, x, w)
    B, Cin, H, W = x.shape
    Cout, _, KH, KW = w.shape
    dx, dw = torch.empty_like(x), torch.empty_like(w)
    ctx = context()
    check(ctx, lib().tb_conv2d_bwd(ctx, _dt(x), _p(dy), _p(x), _p(w), _p(dx), _p(dw), ctypes.c_int(B),
                                   ctypes.c_int(Cin), ctypes.c_int(Cout), ctypes.c_int(H), ctypes.c_int(W),
                                   ctypes.c_int(KH), ctypes.c_int(KW), ctypes.c_int(stride), ctypes.c_int(pad)))
    return dx, dw
