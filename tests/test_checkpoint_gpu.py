"""Checkpoint ingest on the GPU: Llama-layout safetensors files (bf16, and
teeny-quant's int8 with per-channel F32 scales) loaded into the decoder and
checked against the oracle decoder on the same weights."""
import os

import numpy as np
import pytest

import oracle
import st_writer
from decoder_util import SmallCfg
from gpu_util import BF16_TOL, assert_close, dev, no_device_error, np_of, torch
from oracle.decoder import OracleDecoder, random_params

pytestmark = pytest.mark.gpu


def _decoder(cfg, int8):
    from teenygrad_b200.decoder import Decoder, DecoderConfig
    return Decoder(DecoderConfig(n_layers=cfg.n_layers, d_model=cfg.d_model, n_heads=cfg.n_heads,
                                 n_kv_heads=cfg.n_kv_heads, head_dim=cfg.head_dim, ffn_hidden=cfg.ffn_hidden,
                                 vocab=cfg.vocab, rope_theta=cfg.rope_theta, norm_eps=cfg.norm_eps, max_batch=2,
                                 max_seq=64, weights_int8=int8))


def _tensors(cfg, p, int8, tie=False):
    t = {}

    def put(name, a, quant):
        if quant:
            q, s = oracle.quantize_int8(a)
            t[name] = q
            t[name + "_scale"] = s
        else:
            t[name] = ("BF16", oracle.bf16_bits(a))

    put("model.embed_tokens.weight", p["embed"], int8)   # teeny-quant quantises every rank-2 tensor
    if not tie:
        put("lm_head.weight", p["lm_head"], int8)
    t["model.norm.weight"] = p["final_norm"].astype(np.float32)
    for l, L in enumerate(p["layers"]):
        for k, name in st_writer.llama_names(cfg, l).items():
            if L[k].ndim == 1:
                t[name] = L[k].astype(np.float32)
            else:
                put(name, L[k], int8)
    return t


def _check(dec, ora, cfg):
    ids = np.random.default_rng(1).integers(0, cfg.vocab, (2, 12)).astype(np.int32)
    _, logits = dec.prefill(torch.from_numpy(ids).cuda(), return_logits=True)
    ref = ora.forward(ids)
    assert_close(np_of(logits), ref, BF16_TOL, "prefill")
    tok = np.argmax(ref, axis=1).astype(np.int32)
    _, logits = dec.decode_step(torch.from_numpy(tok).cuda(), return_logits=True)
    assert_close(np_of(logits), ora.forward(tok[:, None]), BF16_TOL, "decode")
    no_device_error()


@pytest.mark.parametrize("tie", [False, True])
def test_load_bf16_checkpoint(tmp_path, tie):
    dev()
    cfg = SmallCfg()
    p = random_params(cfg, seed=21)
    if tie:
        p["lm_head"] = p["embed"]
    path = os.path.join(tmp_path, "model.safetensors")
    st_writer.write(path, _tensors(cfg, p, False, tie))
    dec = _decoder(cfg, False)
    dec.load_checkpoint(path)
    _check(dec, OracleDecoder(cfg, p), cfg)


def test_load_teeny_quant_int8_checkpoint(tmp_path):
    dev()
    cfg = SmallCfg()
    p = random_params(cfg, seed=22)
    path = os.path.join(tmp_path, "model-int8.safetensors")
    st_writer.write(path, _tensors(cfg, p, True), {"quantization_config": '{"format": "int-quantized"}'})
    dec = _decoder(cfg, True)
    dec.load_checkpoint(path)
    # the file's int8 embedding is dequantised (q * scale) into the bf16 table
    q, s = oracle.quantize_int8(p["embed"])
    p2 = dict(p, embed=oracle.round_bf16(oracle.dequantize_int8(q, s)))
    _check(dec, OracleDecoder(cfg, p2, int8=True), cfg)


def test_checkpoint_errors(tmp_path):
    dev()
    from teenygrad_b200 import TeenyError
    cfg = SmallCfg()
    p = random_params(cfg, seed=23)
    t = _tensors(cfg, p, True)
    path = os.path.join(tmp_path, "bad.safetensors")
    # int8 weights into a decoder without int8 weights
    st_writer.write(path, t)
    with pytest.raises(TeenyError):
        _decoder(cfg, False).load_checkpoint(path)
    # asymmetric int8 (a zero point) is refused
    t2 = dict(t)
    t2["model.layers.0.self_attn.q_proj.weight_zero_point"] = np.zeros(cfg.n_heads * cfg.head_dim, np.int32)
    st_writer.write(path, t2)
    with pytest.raises(TeenyError):
        _decoder(cfg, True).load_checkpoint(path)
    # a missing tensor
    t3 = dict(t)
    del t3["model.layers.1.mlp.down_proj.weight"]
    st_writer.write(path, t3)
    with pytest.raises(TeenyError):
        _decoder(cfg, True).load_checkpoint(path)
