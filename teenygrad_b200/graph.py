"""Lowering of an op graph onto the library's graph executor (tb_graph_*).

A Graph records ops named after the reference's graph IR
(core/teeny-core/src/graph/mod.rs: Op::Linear :189, LayerNorm :241,
RmsNorm :250, Conv2d :326, Relu :639, Gelu :653, Sigmoid :701, Silu :703,
Add :732, Mul :829, Gather :910, MatMul :1019, ArgMax :1177,
MultiHeadAttention :1241, RotaryEmbedding :1425), then `compile()` lowers
them, the way TritonLowering::lower_with_mapping (kernels/teeny-kernels/src/
graph/mod.rs:689) turns a Graph into kernels: Mul(Silu(g), u) becomes one
SwiGLU node, everything else maps one to one onto a node kind of the
executor.  The reference's RmsNorm RuntimeOp is a stub (graph/mod.rs:454) and
its RotaryEmbedding / MultiHeadAttention / Gather / ArgMax lowerings are TODOs
(:2472-2530, :2250); here they lower like the rest.

    g = Graph()
    x = g.input((1, 128, 256))
    h = g.rms_norm(x, g.param(w_norm), eps=1e-6)
    ...
    g.output(y); g.compile(capture=True)
    (y_out,) = g.run(x_tensor)

The compiled graph plans every input and intermediate into one device arena
(allocated once) and runs stream-ordered on the current torch stream, as one
CUDA graph when capture=True.
"""
from __future__ import annotations

import ctypes

import torch

from ._lib import TB_ACT, TB_BF16, TB_F32, TB_I32, TeenyError, check, lib
from .ops import context

_DT = {torch.float32: TB_F32, torch.bfloat16: TB_BF16, torch.int32: TB_I32}
_TD = {v: k for k, v in _DT.items()}
G_LINEAR, G_MATMUL, G_RMSNORM, G_LAYERNORM, G_ACT, G_ADD, G_SWIGLU = 0, 1, 2, 3, 4, 5, 6
G_ATTENTION, G_ROPE, G_GATHER, G_ARGMAX, G_CONV2D, G_BATCHNORM = 7, 8, 9, 10, 11, 12


class _Attr(ctypes.Structure):
    _fields_ = [("eps", ctypes.c_float), ("act", ctypes.c_int), ("heads", ctypes.c_int), ("kv_heads", ctypes.c_int),
                ("causal", ctypes.c_int), ("scale", ctypes.c_float), ("theta", ctypes.c_float),
                ("stride", ctypes.c_int), ("pad", ctypes.c_int)]


class Value:
    """A tensor of the recorded graph."""

    def __init__(self, graph, idx, shape, dtype):
        self.graph, self.idx, self.shape, self.dtype = graph, idx, tuple(shape), dtype


class Graph:
    def __init__(self, device: int | None = None):
        self.device = torch.cuda.current_device() if device is None else device
        self.ops = []          # (kind, inputs, attrs, out Value)
        self.values = []
        self.inputs, self.outputs, self.params = [], [], []
        self._h = None

    # ----------------------------------------------------------- recording --
    def _val(self, shape, dtype):
        v = Value(self, len(self.values), shape, dtype)
        self.values.append(v)
        return v

    def input(self, shape, dtype=torch.float32) -> Value:
        v = self._val(shape, dtype)
        self.inputs.append(v)
        self.ops.append(("input", [], {}, v))
        return v

    def param(self, t: torch.Tensor) -> Value:
        if not t.is_cuda:
            raise TeenyError(1, "graph parameters live in device memory")
        t = t.contiguous()
        v = self._val(t.shape, t.dtype)
        self.params.append(t)
        self.ops.append(("param", [], {"tensor": t}, v))
        return v

    def _op(self, kind, ins, shape, dtype, **attrs):
        v = self._val(shape, dtype)
        self.ops.append((kind, ins, attrs, v))
        return v

    def linear(self, x, w, bias=None, residual=None):
        return self._op("Linear", [x, w, bias, residual], x.shape[:-1] + (w.shape[0],), x.dtype)

    def matmul(self, a, b):
        return self._op("MatMul", [a, b], a.shape[:-1] + (b.shape[1],), a.dtype)

    def rms_norm(self, x, w, eps=1e-8):
        return self._op("RmsNorm", [x, w], x.shape, x.dtype, eps=eps)

    def layer_norm(self, x, w, b, eps=1e-5):
        return self._op("LayerNorm", [x, w, b], x.shape, x.dtype, eps=eps)

    def silu(self, x):
        return self._op("Silu", [x], x.shape, x.dtype)

    def gelu(self, x):
        return self._op("Gelu", [x], x.shape, x.dtype)

    def relu(self, x):
        return self._op("Relu", [x], x.shape, x.dtype)

    def sigmoid(self, x):
        return self._op("Sigmoid", [x], x.shape, x.dtype)

    def add(self, a, b):
        return self._op("Add", [a, b], a.shape, a.dtype)

    def mul(self, a, b):
        return self._op("Mul", [a, b], a.shape, a.dtype)

    def multi_head_attention(self, q, k=None, v=None, heads=1, kv_heads=None, causal=True, scale=0.0):
        """q, k, v token-major [B, S, H * D]; or q alone as the fused projection
        [B, S, (heads + 2 kv_heads) * D] (k = v = None)."""
        kvh = kv_heads or heads
        if k is None:
            D = q.shape[-1] // (heads + 2 * kvh)
            return self._op("MultiHeadAttention", [q], q.shape[:-1] + (heads * D,), q.dtype, heads=heads,
                            kv_heads=kvh, causal=int(causal), scale=scale)
        return self._op("MultiHeadAttention", [q, k, v], q.shape, q.dtype, heads=heads, kv_heads=kvh,
                        causal=int(causal), scale=scale)

    def rotary_embedding(self, x, pos, theta=10000.0):
        return self._op("RotaryEmbedding", [x, pos], x.shape, x.dtype, theta=theta)

    def gather(self, table, ids):
        return self._op("Gather", [table, ids], ids.shape + (table.shape[1],), table.dtype)

    def argmax(self, x):
        return self._op("ArgMax", [x], x.shape[:-1] or (1,), torch.int32)

    def conv2d(self, x, w, bias=None, bn_scale=None, bn_shift=None, stride=1, pad=0, act=None):
        B, C, H, W = x.shape
        OH = (H + 2 * pad - w.shape[2]) // stride + 1
        OW = (W + 2 * pad - w.shape[3]) // stride + 1
        return self._op("Conv2d", [x, w, bias, bn_scale, bn_shift], (B, w.shape[0], OH, OW), x.dtype, stride=stride,
                        pad=pad, act=-1 if act is None else TB_ACT[act])

    def batch_norm(self, x, gamma, beta, mean, var, eps=1e-5):
        return self._op("BatchNorm", [x, gamma, beta, mean, var], x.shape, x.dtype, eps=eps)

    def output(self, *vals):
        self.outputs.extend(vals)

    # ------------------------------------------------------------ lowering --
    def _uses(self):
        n = {}
        for kind, ins, _, _ in self.ops:
            for v in ins:
                if v is not None:
                    n[v.idx] = n.get(v.idx, 0) + 1
        for v in self.outputs:
            n[v.idx] = n.get(v.idx, 0) + 1
        return n

    def compile(self, capture: bool = True):
        """Lowers the recorded ops onto tb_graph nodes and plans the arena."""
        ctx = context(self.device)
        l = lib()
        h = ctypes.c_void_p()
        check(ctx, l.tb_graph_create(ctx, ctypes.byref(h)))
        self._h = h
        uses = self._uses()
        producer = {v.idx: (kind, ins) for kind, ins, _, v in self.ops}
        tid = {}

        def shape_arr(shape):
            return (ctypes.c_int64 * len(shape))(*shape)

        def node(op, ins, attr, v):
            arr = (ctypes.c_int * len(ins))(*[(-1 if x is None else tid[x.idx]) for x in ins])
            out = ctypes.c_int(0)
            check(ctx, l.tb_graph_node(h, ctypes.c_int(op), arr, ctypes.c_int(len(ins)), ctypes.byref(attr),
                                       ctypes.byref(out)))
            tid[v.idx] = out.value

        fused = set()   # Silu outputs folded into a SwiGLU
        for kind, ins, attrs, v in self.ops:
            if kind == "Mul":
                a, b = ins
                pa = producer.get(a.idx)
                if pa and pa[0] == "Silu" and uses.get(a.idx, 0) == 1:
                    fused.add(a.idx)
        act = {"Silu": TB_ACT["silu"], "Gelu": TB_ACT["gelu_tanh"], "Relu": TB_ACT["relu"], "Sigmoid": TB_ACT["sigmoid"]}
        for kind, ins, attrs, v in self.ops:
            a = _Attr()
            if kind == "input":
                i = ctypes.c_int(0)
                check(ctx, l.tb_graph_input(h, ctypes.c_int(_DT[v.dtype]), ctypes.c_int(len(v.shape)), shape_arr(v.shape),
                                            ctypes.byref(i)))
                tid[v.idx] = i.value
            elif kind == "param":
                t = attrs["tensor"]
                i = ctypes.c_int(0)
                check(ctx, l.tb_graph_param(h, ctypes.c_int(_DT[t.dtype]), ctypes.c_int(max(t.dim(), 1)),
                                            shape_arr(tuple(t.shape) or (1,)), ctypes.c_void_p(t.data_ptr()),
                                            ctypes.byref(i)))
                tid[v.idx] = i.value
            elif kind == "Linear":
                x, w, b, r = ins
                node(G_LINEAR, [x, w, b, r], a, v)
            elif kind == "MatMul":
                node(G_MATMUL, ins, a, v)
            elif kind in ("RmsNorm", "LayerNorm"):
                a.eps = attrs["eps"]
                node(G_RMSNORM if kind == "RmsNorm" else G_LAYERNORM, ins, a, v)
            elif kind in act:
                if v.idx in fused:
                    continue
                a.act = act[kind]
                node(G_ACT, ins, a, v)
            elif kind == "Add":
                node(G_ADD, ins, a, v)
            elif kind == "Mul":
                x, u = ins
                if x.idx not in fused:
                    raise TeenyError(5, "Mul lowers only as the SwiGLU pattern Mul(Silu(gate), up)")
                node(G_SWIGLU, [producer[x.idx][1][0], u], a, v)
            elif kind == "MultiHeadAttention":
                a.heads, a.kv_heads, a.causal, a.scale = attrs["heads"], attrs["kv_heads"], attrs["causal"], attrs["scale"]
                node(G_ATTENTION, ins, a, v)
            elif kind == "RotaryEmbedding":
                a.theta = attrs["theta"]
                node(G_ROPE, ins, a, v)
            elif kind == "Gather":
                node(G_GATHER, ins, a, v)
            elif kind == "ArgMax":
                node(G_ARGMAX, ins, a, v)
            elif kind == "Conv2d":
                a.stride, a.pad, a.act = attrs["stride"], attrs["pad"], attrs["act"]
                node(G_CONV2D, ins, a, v)
            elif kind == "BatchNorm":
                a.eps = attrs["eps"]
                node(G_BATCHNORM, ins, a, v)
            else:
                raise TeenyError(5, f"no lowering for {kind}")
        for o in self.outputs:
            check(ctx, l.tb_graph_mark_output(h, ctypes.c_int(tid[o.idx])))
        check(ctx, l.tb_graph_plan(h, ctypes.c_int(int(capture))))
        self._tid = tid
        return self

    def arena_bytes(self) -> int:
        n = ctypes.c_size_t(0)
        check(None, lib().tb_graph_arena_bytes(self._h, ctypes.byref(n)))
        return n.value

    # ------------------------------------------------------------- running --
    def run(self, *inputs):
        """inputs: torch tensors (host or device) in input() order; returns new
        device tensors holding the outputs."""
        if self._h is None:
            raise TeenyError(1, "compile() first")
        ctx = context(self.device)
        l = lib()
        for v, t in zip(self.inputs, inputs):
            t = t.to(v.dtype).contiguous()
            check(ctx, l.tb_graph_write(self._h, ctypes.c_int(self._tid[v.idx]), ctypes.c_void_p(t.data_ptr()),
                                        ctypes.c_size_t(t.numel() * t.element_size())))
        check(ctx, l.tb_graph_run(self._h))
        outs = []
        for v in self.outputs:
            o = torch.empty(v.shape, dtype=v.dtype, device=torch.device("cuda", self.device))
            check(ctx, l.tb_graph_read(self._h, ctypes.c_int(self._tid[v.idx]), ctypes.c_void_p(o.data_ptr()),
                                       ctypes.c_size_t(o.numel() * o.element_size())))
            outs.append(o)
        return outs

    def launch(self):
        """The node launches only (inputs already written), on the current stream."""
        ctx = context(self.device)
        check(ctx, lib().tb_graph_run(self._h))

    def close(self):
        if self._h is not None:
            lib().tb_graph_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
