"""CPU oracle of the Llama-style decoder -- TEST INFRASTRUCTURE ONLY.

Composes the oracle's restated primitives exactly as the B200 executor
composes its kernels, with the same bf16 rounding points (every activation
tensor that the GPU stores in bf16 is rounded to bf16 here):

    x = embed[ids]
    per layer:  h = rmsnorm(x); qkv = h Wqkv^T; q, k = rope(q, k); cache k, v
                a = attention(q, cache) (causal, GQA); x = x + a Wo^T
                h = rmsnorm(x); x = x + swiglu(h Wg^T, h Wu^T) Wd^T
    logits = rmsnorm(x_last) lm_head^T (f32); next = argmax(logits)

The reference has no such model (apps/teeny-llm is a placeholder) and its
graph lowering lacks attention, RoPE and gather (kernels/teeny-kernels/src/
graph/mod.rs:2472-2530); each step follows the primitive it names, whose
reference citation is in oracle.c.  int8 mode replaces every linear layer by
int8_linear on quantize_int8 weights (teeny-quant affine.rs:55-148).
"""
from __future__ import annotations

import numpy as np

from . import (argmax, attention, int8_linear, linear, quantize_int8, rmsnorm, rope, round_bf16,
               swiglu)


class OracleDecoder:
    def __init__(self, cfg, params, int8=False):
        """params: dict with 'embed', 'lm_head', 'final_norm' and per layer
        'layers': [ {attn_norm, wq, wk, wv, wo, mlp_norm, w_gate, w_up, w_down} ]
        (f32 arrays, already on the bf16 grid)."""
        self.c = cfg
        self.p = params
        self.int8 = int8
        self.q = {}
        if int8:
            for i, L in enumerate(params["layers"]):
                for k in ("wq", "wk", "wv", "wo", "w_gate", "w_up", "w_down"):
                    self.q[(i, k)] = quantize_int8(L[k])
            self.q[(-1, "lm_head")] = quantize_int8(params["lm_head"])
        self.k = None
        self.v = None
        self.len = 0

    def _lin(self, x, layer, name, resid=None):
        if self.int8:
            q, s = self.q[(layer, name)]
            return int8_linear(x, q, s, resid)
        w = self.p["lm_head"] if layer < 0 else self.p["layers"][layer][name]
        return linear(x, w, None, resid)

    def forward(self, ids):
        """ids [B, S] int -> f32 logits [B, V] of the last position; appends to the cache."""
        c = self.c
        B, S = ids.shape
        hd, Hq, Hkv = c.head_dim, c.n_heads, c.n_kv_heads
        if self.k is None:
            self.k = np.zeros((c.n_layers, B, Hkv, 0, hd), np.float32)
            self.v = np.zeros((c.n_layers, B, Hkv, 0, hd), np.float32)
        pos0 = self.len
        T = B * S
        x = self.p["embed"][ids.reshape(-1)].astype(np.float32)
        pos = np.tile(np.arange(pos0, pos0 + S, dtype=np.int32), B)
        newk, newv = [], []
        for l, L in enumerate(self.p["layers"]):
            h = round_bf16(rmsnorm(x, L["attn_norm"], c.norm_eps)[0])
            qkv = np.concatenate([round_bf16(self._lin(h, l, n)) for n in ("wq", "wk", "wv")], axis=1)
            q = qkv[:, :Hq * hd].reshape(T, Hq, hd)
            k = qkv[:, Hq * hd:(Hq + Hkv) * hd].reshape(T, Hkv, hd)
            v = qkv[:, (Hq + Hkv) * hd:].reshape(T, Hkv, hd)
            q = round_bf16(rope(q, pos, c.rope_theta))
            k = round_bf16(rope(k, pos, c.rope_theta))
            kb = k.reshape(B, S, Hkv, hd).transpose(0, 2, 1, 3)
            vb = v.reshape(B, S, Hkv, hd).transpose(0, 2, 1, 3)
            kc = np.concatenate([self.k[l], kb], axis=2)
            vc = np.concatenate([self.v[l], vb], axis=2)
            newk.append(kc)
            newv.append(vc)
            qb = q.reshape(B, S, Hq, hd).transpose(0, 2, 1, 3)
            o, _ = attention(qb, kc, vc, 1.0 / np.sqrt(hd), True)
            a = round_bf16(o.transpose(0, 2, 1, 3).reshape(T, Hq * hd))
            x = round_bf16(self._lin(a, l, "wo", resid=x))
            h = round_bf16(rmsnorm(x, L["mlp_norm"], c.norm_eps)[0])
            g = self._lin(h, l, "w_gate")
            u = self._lin(h, l, "w_up")
            act = round_bf16(swiglu(g, u))
            x = round_bf16(self._lin(act, l, "w_down", resid=x))
        self.k = np.stack(newk)
        self.v = np.stack(newv)
        self.len += S
        last = x.reshape(B, S, -1)[:, -1, :]
        hl = round_bf16(rmsnorm(last, self.p["final_norm"], c.norm_eps)[0])
        logits = self._lin(hl, -1, "lm_head")
        return logits

    @staticmethod
    def greedy(logits):
        return argmax(logits)


def random_params(cfg, seed=0, std=0.02):
    """bf16-grid f32 parameters, N(0, std) weights, norm gains ~ U(0.8, 1.2)."""
    r = np.random.default_rng(seed)
    d, F, V = cfg.d_model, cfg.ffn_hidden, cfg.vocab
    qd, kd = cfg.n_heads * cfg.head_dim, cfg.n_kv_heads * cfg.head_dim

    def w(*shape):
        return round_bf16((r.standard_normal(shape) * std).astype(np.float32))

    def g(n):
        return round_bf16(r.uniform(0.8, 1.2, n).astype(np.float32))

    layers = []
    for _ in range(cfg.n_layers):
        layers.append(dict(attn_norm=g(d), wq=w(qd, d), wk=w(kd, d), wv=w(kd, d), wo=w(d, qd), mlp_norm=g(d),
                           w_gate=w(F, d), w_up=w(F, d), w_down=w(d, F)))
    return dict(embed=round_bf16(r.standard_normal((V, d)).astype(np.float32)), lm_head=w(V, d),
                final_norm=g(d), layers=layers)


def block_forward(x, p, n_heads, eps=1e-6):
    """CPU oracle of the fp32 pre-norm block (teenygrad_b200.block), numpy f32."""
    B, S, d = x.shape
    hd = d // n_heads
    X = x.reshape(B * S, d)
    h = rmsnorm(X, p["attn_norm"], eps)[0]
    q, k, v = (linear(h, p[n]) for n in ("wq", "wk", "wv"))

    def heads(t):
        return t.reshape(B, S, n_heads, hd).transpose(0, 2, 1, 3)

    o, _ = attention(heads(q), heads(k), heads(v), 1.0 / np.sqrt(hd), True)
    o = o.transpose(0, 2, 1, 3).reshape(B * S, d)
    X = linear(o, p["wo"], None, X)
    h = rmsnorm(X, p["mlp_norm"], eps)[0]
    a = swiglu(linear(h, p["w_gate"]), linear(h, p["w_up"]))
    return linear(a, p["w_down"], None, X).reshape(B, S, d)
