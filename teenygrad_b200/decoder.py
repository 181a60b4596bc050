"""Llama-style decoder on the C-ABI executor (tb_decoder_*).

    dec = Decoder(DecoderConfig.llama_1b(max_batch=16, max_seq=1152))
    dec.init_random(seed=0)
    out = dec.generate(prompt_ids_cuda_int32, n_new=128)   # [B, n_new] int32

Parameters live inside the executor in its own layout (fused QKV rows,
gate/up interleaved for the SwiGLU epilogue); set_param accepts the PyTorch
layout of each tensor.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from ._lib import TB_BF16, TB_F32, TeenyError, check, lib
from .ops import context

P_EMBED, P_ATTN_NORM, P_WQ, P_WK, P_WV, P_WO, P_MLP_NORM = 0, 1, 2, 3, 4, 5, 6
P_W_GATE, P_W_UP, P_W_DOWN, P_FINAL_NORM, P_LM_HEAD = 7, 8, 9, 10, 11


class _Cfg(ctypes.Structure):
    _fields_ = [("n_layers", ctypes.c_int), ("d_model", ctypes.c_int), ("n_heads", ctypes.c_int),
                ("n_kv_heads", ctypes.c_int), ("head_dim", ctypes.c_int), ("ffn_hidden", ctypes.c_int),
                ("vocab", ctypes.c_int), ("rope_theta", ctypes.c_float), ("norm_eps", ctypes.c_float),
                ("max_batch", ctypes.c_int), ("max_seq", ctypes.c_int), ("max_prefill_tokens", ctypes.c_int),
                ("weights_int8", ctypes.c_int)]


@dataclass
class DecoderConfig:
    n_layers: int = 16
    d_model: int = 2048
    n_heads: int = 32
    n_kv_heads: int = 8
    head_dim: int = 64
    ffn_hidden: int = 8192
    vocab: int = 32000
    rope_theta: float = 10000.0
    norm_eps: float = 1e-5
    max_batch: int = 16
    max_seq: int = 1152
    max_prefill_tokens: int = 0
    weights_int8: bool = False

    @classmethod
    def llama_1b(cls, **kw):
        return cls(**kw)

    def _c(self):
        return _Cfg(self.n_layers, self.d_model, self.n_heads, self.n_kv_heads, self.head_dim, self.ffn_hidden,
                    self.vocab, self.rope_theta, self.norm_eps, self.max_batch, self.max_seq,
                    self.max_prefill_tokens, int(self.weights_int8))


class Decoder:
    def __init__(self, cfg: DecoderConfig, device: int | None = None):
        self.cfg = cfg
        self.device = torch.cuda.current_device() if device is None else device
        self.ctx = context(self.device)
        self._h = ctypes.c_void_p()
        c = cfg._c()
        check(self.ctx, lib().tb_decoder_create(self.ctx, ctypes.byref(c), ctypes.byref(self._h)))
        self.B = 0

    def close(self):
        if self._h:
            lib().tb_decoder_destroy(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _ctx(self):
        return context(self.device)

    # ---------------------------------------------------------- params --
    def set_param(self, kind: int, tensor, layer: int = 0):
        """tensor: numpy f32 (host) or torch f32/bf16 (host or device), PyTorch layout."""
        import numpy as np
        keep = tensor
        if isinstance(tensor, np.ndarray):
            keep = np.ascontiguousarray(tensor, dtype=np.float32)
            ptr, dt, host = keep.ctypes.data, TB_F32, 1
        else:
            keep = tensor.contiguous()
            if keep.dtype not in (torch.float32, torch.bfloat16):
                keep = keep.float()
            ptr = keep.data_ptr()
            dt = TB_F32 if keep.dtype == torch.float32 else TB_BF16
            host = 0 if keep.is_cuda else 1
        self._ctx()
        check(self.ctx, lib().tb_decoder_set_param(self._h, ctypes.c_int(layer), ctypes.c_int(kind),
                                                   ctypes.c_void_p(ptr), ctypes.c_int(dt), ctypes.c_int(host)))

    def set_param_int8(self, kind: int, q, scale, layer: int = 0):
        """int8 weight [rows, cols] + f32 scale [rows] (teeny-quant's I8 + _scale), numpy or torch."""
        import numpy as np
        if isinstance(q, np.ndarray):
            qk, sk = np.ascontiguousarray(q, np.int8), np.ascontiguousarray(scale, np.float32)
            qp, sp, host = qk.ctypes.data, sk.ctypes.data, 1
        else:
            qk, sk = q.contiguous(), scale.float().contiguous()
            qp, sp, host = qk.data_ptr(), sk.data_ptr(), 0 if qk.is_cuda else 1
        self._ctx()
        check(self.ctx, lib().tb_decoder_set_param_int8(self._h, ctypes.c_int(layer), ctypes.c_int(kind),
                                                        ctypes.c_void_p(qp), ctypes.c_void_p(sp), ctypes.c_int(host)))

    def load_checkpoint(self, path: str):
        """Loads a Llama-layout .safetensors checkpoint (F32 / BF16, or teeny-quant
        int8 with per-channel scales) and prepares the decoder."""
        from .checkpoint import SafeTensors
        with SafeTensors(path) as st:
            self._ctx()
            check(self.ctx, lib().tb_decoder_load_safetensors(self._h, st._h))

    def init_random(self, seed: int = 0, std: float = 0.02):
        self._ctx()
        check(self.ctx, lib().tb_decoder_init_random(self._h, ctypes.c_uint64(seed), ctypes.c_float(std)))
        self.prepare()

    def prepare(self):
        self._ctx()
        check(self.ctx, lib().tb_decoder_prepare(self._h))

    # --------------------------------------------------------- running --
    def prefill(self, ids: torch.Tensor, return_logits: bool = False):
        """ids: cuda int32 [B, S].  Returns next token ids [B] (and f32 logits [B, V])."""
        assert ids.is_cuda and ids.dtype == torch.int32
        ids = ids.contiguous()
        B, S = ids.shape
        self._ctx()
        nxt = torch.empty(B, device=ids.device, dtype=torch.int32)
        logits = torch.empty(B, self.cfg.vocab, device=ids.device, dtype=torch.float32) if return_logits else None
        check(self.ctx, lib().tb_decoder_prefill(self._h, ctypes.c_void_p(ids.data_ptr()), ctypes.c_int(B),
                                                 ctypes.c_int(S), ctypes.c_void_p(0 if logits is None else logits.data_ptr()),
                                                 ctypes.c_void_p(nxt.data_ptr())))
        self.B = B
        return (nxt, logits) if return_logits else nxt

    def decode_step(self, ids: torch.Tensor | None = None, return_logits: bool = False):
        self._ctx()
        dev = torch.device("cuda", self.device)
        nxt = torch.empty(self.B, device=dev, dtype=torch.int32)
        logits = torch.empty(self.B, self.cfg.vocab, device=dev, dtype=torch.float32) if return_logits else None
        if ids is not None:
            ids = ids.to(torch.int32).contiguous()
        check(self.ctx, lib().tb_decoder_decode_step(self._h, ctypes.c_void_p(0 if ids is None else ids.data_ptr()),
                                                     ctypes.c_void_p(0 if logits is None else logits.data_ptr()),
                                                     ctypes.c_void_p(nxt.data_ptr())))
        return (nxt, logits) if return_logits else nxt

    def generate(self, prompt_ids: torch.Tensor, n_new: int, out: torch.Tensor | None = None) -> torch.Tensor:
        assert prompt_ids.is_cuda and prompt_ids.dtype == torch.int32
        prompt_ids = prompt_ids.contiguous()
        B, S = prompt_ids.shape
        if out is None:
            out = torch.empty(B, n_new, device=prompt_ids.device, dtype=torch.int32)
        self._ctx()
        check(self.ctx, lib().tb_decoder_generate(self._h, ctypes.c_void_p(prompt_ids.data_ptr()), ctypes.c_int(B),
                                                  ctypes.c_int(S), ctypes.c_int(n_new), ctypes.c_void_p(out.data_ptr())))
        self.B = B
        return out

    def fill_kv_random(self, ids: torch.Tensor, length: int, seed: int = 0):
        """Decode-only workloads: KV cache of len(ids) sequences pre-filled with
        `length` positions of N(0,1); ids [B] are the current tokens."""
        ids = ids.to(torch.int32).contiguous()
        self._ctx()
        check(self.ctx, lib().tb_decoder_fill_kv_random(self._h, ctypes.c_int(ids.numel()), ctypes.c_int(length),
                                                        ctypes.c_uint64(seed), ctypes.c_void_p(ids.data_ptr())))
        self.B = ids.numel()

    def read_kv(self, layer: int, batch: int, length: int):
        """Copies of the cached keys and values of `layer`: bf16 [batch, n_kv_heads,
        length, head_dim] each (positions [0, length) of the first `batch` sequences)."""
        c = self.cfg
        dev = torch.device("cuda", self.device)
        k = torch.empty(batch, c.n_kv_heads, length, c.head_dim, device=dev, dtype=torch.bfloat16)
        v = torch.empty_like(k)
        self._ctx()
        check(self.ctx, lib().tb_decoder_read_kv(self._h, ctypes.c_int(layer), ctypes.c_int(batch),
                                                 ctypes.c_int(length), ctypes.c_void_p(k.data_ptr()),
                                                 ctypes.c_void_p(v.data_ptr())))
        torch.cuda.current_stream(dev).synchronize()
        return k, v

    def seq_len(self) -> int:
        n = ctypes.c_int(0)
        check(self.ctx, lib().tb_decoder_seq_len(self._h, ctypes.byref(n)))
        return n.value


__all__ = ["Decoder", "DecoderConfig", "TeenyError"]
