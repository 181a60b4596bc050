"""Shared small decoder configuration and parameter upload for the tests."""
from dataclasses import dataclass

import numpy as np


@dataclass
class SmallCfg:
    n_layers: int = 2
    d_model: int = 256
    n_heads: int = 4
    n_kv_heads: int = 2
    head_dim: int = 64
    ffn_hidden: int = 512
    vocab: int = 1000
    rope_theta: float = 10000.0
    norm_eps: float = 1e-5


def upload(dec, params):
    from teenygrad_b200 import decoder as D
    dec.set_param(D.P_EMBED, params["embed"])
    dec.set_param(D.P_LM_HEAD, params["lm_head"])
    dec.set_param(D.P_FINAL_NORM, params["final_norm"])
    names = [("attn_norm", D.P_ATTN_NORM), ("wq", D.P_WQ), ("wk", D.P_WK), ("wv", D.P_WV), ("wo", D.P_WO),
             ("mlp_norm", D.P_MLP_NORM), ("w_gate", D.P_W_GATE), ("w_up", D.P_W_UP), ("w_down", D.P_W_DOWN)]
    for i, L in enumerate(params["layers"]):
        for n, k in names:
            dec.set_param(k, L[n], layer=i)
    dec.prepare()
