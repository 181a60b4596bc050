"""CPU oracle for the teenygrad hot path -- TEST INFRASTRUCTURE ONLY.

ctypes + numpy wrapper around ``oracle.c`` (a C restatement of the reference
kernels' arithmetic, each function citing the reference file:line it follows).
Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg
may import this package, and only as the checker or the timed CPU baseline;
the product library ``teenygrad_b200`` never imports it.

The shared library is built by :func:`build` (``gcc -O3 -fopenmp``) into
``oracle/liboracle.so`` and rebuilt on demand if it is missing.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "oracle.c")
LIB = os.path.join(HERE, "liboracle.so")

# -march=x86-64-v3 (AVX2/FMA) rather than -march=native: the library is built
# in one container and run on another host.  -ffp-contract=off keeps every
# float operation individually rounded (the int8 quantiser is bit-exact).
CFLAGS = ["-O3", "-march=x86-64-v3", "-ffp-contract=off", "-fopenmp", "-fPIC", "-shared"]


def build(force: bool = False) -> str:
    if force or not os.path.exists(LIB) or os.path.getmtime(LIB) < os.path.getmtime(SRC):
        tmp = LIB + f".tmp{os.getpid()}"
        subprocess.check_call(["gcc", *CFLAGS, SRC, "-o", tmp, "-lm"])
        os.replace(tmp, LIB)
    return LIB


_lib = None

_F = ctypes.POINTER(ctypes.c_float)
_I64 = ctypes.c_int64


def lib():
    global _lib
    if _lib is None:
        _lib = ctypes.CDLL(build())
        _lib.or_f32_to_bf16.restype = ctypes.c_uint16
        _lib.or_f32_to_bf16.argtypes = [ctypes.c_float]
        _lib.or_num_threads.restype = ctypes.c_int
    return _lib


def _p(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def _f32(a):
    return None if a is None else np.ascontiguousarray(a, dtype=np.float32)


# --------------------------------------------------------------- bf16 -----

def bf16_bits(x) -> np.ndarray:
    """f32 -> bf16 bit patterns (uint16), round-to-nearest-even."""
    x = _f32(x)
    out = np.empty(x.shape, dtype=np.uint16)
    lib().or_f32_to_bf16_array(_p(x), _p(out), _I64(x.size))
    return out


def bf16_to_f32(bits) -> np.ndarray:
    bits = np.ascontiguousarray(bits, dtype=np.uint16)
    out = np.empty(bits.shape, dtype=np.float32)
    lib().or_bf16_to_f32_array(_p(bits), _p(out), _I64(bits.size))
    return out


def round_bf16(x) -> np.ndarray:
    """Round an f32 array to the nearest bf16 value, returned as f32."""
    return bf16_to_f32(bf16_bits(x))


def num_threads() -> int:
    return lib().or_num_threads()


def set_num_threads(n: int) -> None:
    lib().or_set_num_threads(ctypes.c_int(n))


# -------------------------------------------------------------- ops -------

def rmsnorm(x, w, eps):
    x, w = _f32(x), _f32(w)
    M, N = x.shape
    y = np.empty_like(x)
    rrms = np.empty(M, np.float32)
    lib().or_rmsnorm(_p(x), _p(w), _p(y), _p(rrms), _I64(M), _I64(N), ctypes.c_float(eps))
    return y, rrms


def layernorm(x, w, b, eps):
    x, w, b = _f32(x), _f32(w), _f32(b)
    M, N = x.shape
    y = np.empty_like(x)
    lib().or_layernorm(_p(x), _p(w), _p(b), _p(y), _I64(M), _I64(N), ctypes.c_float(eps))
    return y


ACT = {"silu": 0, "gelu_tanh": 1, "relu": 2, "sigmoid": 3}


def act(kind, x):
    x = _f32(x)
    y = np.empty_like(x)
    lib().or_act(ctypes.c_int(ACT[kind]), _p(x), _p(y), _I64(x.size))
    return y


def swiglu(g, u):
    g, u = _f32(g), _f32(u)
    y = np.empty_like(g)
    lib().or_swiglu(_p(g), _p(u), _p(y), _I64(g.size))
    return y


def add(a, b):
    a, b = _f32(a), _f32(b)
    y = np.empty_like(a)
    lib().or_add(_p(a), _p(b), _p(y), _I64(a.size))
    return y


def linear(x, w, bias=None, resid=None):
    x, w, bias, resid = _f32(x), _f32(w), _f32(bias), _f32(resid)
    M, K = x.shape
    N = w.shape[0]
    y = np.empty((M, N), np.float32)
    lib().or_linear(_p(x), _p(w), _p(bias), _p(resid), _p(y), _I64(M), _I64(N), _I64(K))
    return y


def matmul(a, b):
    a, b = _f32(a), _f32(b)
    M, K = a.shape
    N = b.shape[1]
    c = np.empty((M, N), np.float32)
    lib().or_matmul(_p(a), _p(b), _p(c), _I64(M), _I64(N), _I64(K))
    return c


def attention(q, k, v, scale, causal):
    """q [B,Hq,Sq,D], k/v [B,Hkv,Sk,D] -> (o [B,Hq,Sq,D], lse [B,Hq,Sq])."""
    q, k, v = _f32(q), _f32(k), _f32(v)
    B, Hq, Sq, D = q.shape
    Hkv, Sk = k.shape[1], k.shape[2]
    o = np.empty_like(q)
    lse = np.empty((B, Hq, Sq), np.float32)
    lib().or_attention(_p(q), _p(k), _p(v), _p(o), _p(lse), _I64(B), _I64(Hq), _I64(Hkv),
                       _I64(Sq), _I64(Sk), _I64(D), ctypes.c_float(scale), ctypes.c_int(int(causal)))
    return o, lse


def bn_fold(gamma, beta, mean, var, eps, bias=None):
    gamma, beta, mean, var, bias = map(_f32, (gamma, beta, mean, var, bias))
    C = gamma.size
    sc = np.empty(C, np.float32)
    sh = np.empty(C, np.float32)
    lib().or_bn_fold(_p(gamma), _p(beta), _p(mean), _p(var), _p(bias), ctypes.c_float(eps),
                     _p(sc), _p(sh), _I64(C))
    return sc, sh


CONV_ACT = {None: -1, "silu": 0, "relu": 2}


def conv2d(x, w, bias=None, scale=None, shift=None, stride=1, pad=0, act=None):
    x, w, bias, scale, shift = map(_f32, (x, w, bias, scale, shift))
    B, Cin, H, W = x.shape
    Cout, _, KH, KW = w.shape
    OH = (H + 2 * pad - KH) // stride + 1
    OW = (W + 2 * pad - KW) // stride + 1
    y = np.empty((B, Cout, OH, OW), np.float32)
    lib().or_conv2d(_p(x), _p(w), _p(bias), _p(scale), _p(shift), _p(y), _I64(B), _I64(Cin),
                    _I64(Cout), _I64(H), _I64(W), _I64(KH), _I64(KW), _I64(stride), _I64(pad),
                    ctypes.c_int(CONV_ACT[act]))
    return y


def batchnorm_inference(x, gamma, beta, mean, var, eps):
    x = _f32(x)
    B, C = x.shape[0], x.shape[1]
    HW = int(np.prod(x.shape[2:])) if x.ndim > 2 else 1
    y = np.empty_like(x)
    lib().or_batchnorm_inference(_p(x), _p(_f32(gamma)), _p(_f32(beta)), _p(_f32(mean)),
                                 _p(_f32(var)), _p(y), _I64(B), _I64(C), _I64(HW),
                                 ctypes.c_float(eps))
    return y


def quantize_int8(w):
    w = _f32(w)
    N, K = w.shape
    q = np.empty((N, K), np.int8)
    s = np.empty(N, np.float32)
    lib().or_quantize_int8(_p(w), _p(q), _p(s), _I64(N), _I64(K))
    return q, s


def dequantize_int8(q, s):
    q = np.ascontiguousarray(q, dtype=np.int8)
    s = _f32(s)
    N, K = q.shape
    w = np.empty((N, K), np.float32)
    lib().or_dequantize_int8(_p(q), _p(s), _p(w), _I64(N), _I64(K))
    return w


def int8_linear(x, q, s, resid=None):
    x, s, resid = _f32(x), _f32(s), _f32(resid)
    q = np.ascontiguousarray(q, dtype=np.int8)
    M, K = x.shape
    N = q.shape[0]
    y = np.empty((M, N), np.float32)
    lib().or_int8_linear(_p(x), _p(q), _p(s), _p(resid), _p(y), _I64(M), _I64(N), _I64(K))
    return y


def rope(x, pos, theta):
    """x [T,H,D], pos [T] int32."""
    x = _f32(x)
    pos = np.ascontiguousarray(pos, dtype=np.int32)
    T, H, D = x.shape
    y = np.empty_like(x)
    lib().or_rope(_p(x), _p(pos), _p(y), _I64(T), _I64(H), _I64(D), ctypes.c_float(theta))
    return y


def embedding(table, ids):
    table = _f32(table)
    ids = np.ascontiguousarray(ids, dtype=np.int32)
    y = np.empty((ids.size, table.shape[1]), np.float32)
    lib().or_embedding(_p(table), _p(ids), _p(y), _I64(ids.size), _I64(table.shape[1]))
    return y


def argmax(x):
    x = _f32(x)
    M, N = x.shape
    out = np.empty(M, np.int32)
    lib().or_argmax(_p(x), _p(out), _I64(M), _I64(N))
    return out


def quantize_int8_numpy(w):
    """Independent numpy restatement of quantize_affine (symmetric, per output
    channel, 8 bits; utilities/teeny-quant/src/quant/affine.rs:91-143), used to
    cross-check the C oracle.  Rounding is half away from zero, written as
    sign(t) * floor(|t| + 0.5) -- NOT np.round, which rounds half to even."""
    w = np.asarray(w, dtype=np.float32)
    with np.errstate(invalid="ignore", divide="ignore"):
        # `x < vmin` / `x > vmax` skip NaN (fmin / fmax do too); an all-NaN row
        # keeps the +Inf / -Inf start values
        vmin = np.fmin.reduce(w, axis=1, initial=np.inf)
        vmax = np.fmax.reduce(w, axis=1, initial=-np.inf)
        fin = np.isfinite(vmin)
        lo = np.where(fin, np.minimum(vmin, np.float32(0)), np.float32(0)).astype(np.float32)
        hi = np.where(fin, np.maximum(vmax, np.float32(0)), np.float32(0)).astype(np.float32)
        amax = np.maximum(np.abs(lo), np.abs(hi)).astype(np.float32)
        scale = np.where(amax == 0, np.float32(1), amax / np.float32(127)).astype(np.float32)
        t = (w / scale[:, None]).astype(np.float32)
        # |t| + 0.5 in float64 is exact for any float32 t (no double rounding at
        # the 0.49999997 boundary).
        td = t.astype(np.float64)
        r = np.sign(td) * np.floor(np.abs(td) + 0.5)
        # `as i32` saturates (NaN -> 0) before the clamp to [-127, 127]
        r = np.where(np.isnan(r), 0.0, r)
    q = np.clip(r, -127, 127).astype(np.int8)
    return q, scale


# -------------------------------------------------------------- backward ----
def rmsnorm_bwd(dy, x, w, rrms, dw=None):
    """dx and dw (accumulated into a copy of dw, zeros if None); rmsnorm.rs:125-277."""
    dy, x, w, rrms = map(_f32, (dy, x, w, rrms))
    M, N = x.shape
    dx = np.empty_like(x)
    dwo = np.zeros(N, np.float32) if dw is None else np.array(dw, dtype=np.float32, copy=True)
    lib().or_rmsnorm_bwd(_p(dy), _p(x), _p(w), _p(rrms), _p(dx), _p(dwo), _I64(M), _I64(N))
    return dx, dwo


def linear_bwd(x, w, dy):
    """(dx, dw, db) of y = x w^T + b; linear.rs:119-249."""
    x, w, dy = map(_f32, (x, w, dy))
    M, K = x.shape
    N = w.shape[0]
    dx = np.empty((M, K), np.float32)
    dw = np.empty((N, K), np.float32)
    db = np.empty(N, np.float32)
    lib().or_linear_bwd(_p(x), _p(w), _p(dy), _p(dx), _p(dw), _p(db), _I64(M), _I64(N), _I64(K))
    return dx, dw, db


def attention_bwd(q, k, v, o, do, lse, scale, causal):
    """(dq, dk, dv); flash_attn2.rs:160-447 plus causal / GQA."""
    q, k, v, o, do, lse = map(_f32, (q, k, v, o, do, lse))
    B, Hq, Sq, D = q.shape
    Hkv, Sk = k.shape[1], k.shape[2]
    dq, dk, dv = np.empty_like(q), np.empty_like(k), np.empty_like(v)
    lib().or_attention_bwd(_p(q), _p(k), _p(v), _p(o), _p(do), _p(lse), _p(dq), _p(dk), _p(dv), _I64(B), _I64(Hq),
                           _I64(Hkv), _I64(Sq), _I64(Sk), _I64(D), ctypes.c_float(scale), ctypes.c_int(int(causal)))
    return dq, dk, dv


def conv2d_bwd(dy, x, w, stride=1, pad=0):
    """(dx, dw); conv2d.rs:395-521 (groups = 1)."""
    dy, x, w = map(_f32, (dy, x, w))
    B, Cin, H, W = x.shape
    Cout, _, KH, KW = w.shape
    dx, dw = np.empty_like(x), np.empty_like(w)
    lib().or_conv2d_bwd(_p(dy), _p(x), _p(w), _p(dx), _p(dw), _I64(B), _I64(Cin), _I64(Cout), _I64(H), _I64(W),
                        _I64(KH), _I64(KW), _I64(stride), _I64(pad))
    return dx, dw
