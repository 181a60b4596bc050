"""GPU parity of the decoder executor against the oracle decoder composition.

Logits: bf16 tolerance 2e-2 (normalised max abs error).  Tokens: the greedy
token must match wherever the oracle's top-2 margin exceeds the tolerance.
"""
import numpy as np
import pytest

from decoder_util import SmallCfg, upload
from gpu_util import BF16_TOL, assert_close, dev, no_device_error, np_of, torch
from oracle.decoder import OracleDecoder, random_params

pytestmark = pytest.mark.gpu


def make(cfg, int8=False, max_batch=4, max_seq=160):
    from teenygrad_b200.decoder import Decoder, DecoderConfig
    dc = DecoderConfig(n_layers=cfg.n_layers, d_model=cfg.d_model, n_heads=cfg.n_heads, n_kv_heads=cfg.n_kv_heads,
                       head_dim=cfg.head_dim, ffn_hidden=cfg.ffn_hidden, vocab=cfg.vocab, rope_theta=cfg.rope_theta,
                       norm_eps=cfg.norm_eps, max_batch=max_batch, max_seq=max_seq, weights_int8=int8)
    return Decoder(dc)


def check_tokens(got, logits_ref):
    ref = np.argmax(logits_ref, axis=1)
    srt = np.sort(logits_ref, axis=1)
    margin = srt[:, -1] - srt[:, -2]
    scale = max(1.0, np.abs(logits_ref).max())
    sure = margin > 2 * BF16_TOL * scale
    assert np.array_equal(np.asarray(got)[sure], ref[sure])


# S = 20: 40 prompt tokens take the decode GEMV (RoPE and KV-cache writes in its
# epilogue); S = 70, 129: the tensor-core GEMM and the separate RoPE kernel.
# n_heads = 5, n_kv_heads = 1: q+k+v rows (448) are not a multiple of 256, so the
# QKV weights stay unpermuted and decode uses the separate RoPE kernel too.
@pytest.mark.parametrize("S,heads", [(20, (4, 2)), (70, (4, 2)), (129, (4, 2)), (20, (5, 1)), (70, (5, 1))])
def test_decoder_prefill_and_decode_bf16(S, heads):
    dev()
    cfg = SmallCfg(n_heads=heads[0], n_kv_heads=heads[1])
    p = random_params(cfg, seed=3)
    dec = make(cfg)
    upload(dec, p)
    ora = OracleDecoder(cfg, p)
    ids = np.random.default_rng(S).integers(0, cfg.vocab, (2, S)).astype(np.int32)
    nxt, logits = dec.prefill(torch.from_numpy(ids).cuda(), return_logits=True)
    ref = ora.forward(ids)
    assert_close(np_of(logits), ref, BF16_TOL, "prefill logits")
    check_tokens(nxt.cpu().numpy(), ref)
    for step in range(4):   # teacher-forced on the oracle's greedy tokens
        tok = np.argmax(ref, axis=1).astype(np.int32)
        nxt, logits = dec.decode_step(torch.from_numpy(tok).cuda(), return_logits=True)
        ref = ora.forward(tok[:, None])
        assert_close(np_of(logits), ref, BF16_TOL, f"decode step {step}")
        check_tokens(nxt.cpu().numpy(), ref)
    assert dec.seq_len() == S + 4
    no_device_error()


def test_decoder_generate_matches_stepwise():
    dev()
    cfg = SmallCfg()
    p = random_params(cfg, seed=4)
    dec = make(cfg)
    upload(dec, p)
    ids = torch.from_numpy(np.random.default_rng(9).integers(0, cfg.vocab, (3, 40)).astype(np.int32)).cuda()
    out = dec.generate(ids, n_new=6)
    toks = [dec.prefill(ids)]
    for _ in range(5):
        toks.append(dec.decode_step())
    step = torch.stack(toks, dim=1)
    assert torch.equal(out, step)
    no_device_error()


def test_decoder_generate_long_matches_stepwise():
    """generate() replays a graph of several decode steps (plus single steps for the
    rest): the tokens equal prefill + one decode_step at a time, again on the same
    decoder (the graphs are reused) and at another batch size (rebuilt)."""
    dev()
    cfg = SmallCfg()
    p = random_params(cfg, seed=6)
    dec = make(cfg)
    upload(dec, p)
    rng = np.random.default_rng(10)
    for B, n_new in ((3, 20), (3, 17), (2, 9)):
        ids = torch.from_numpy(rng.integers(0, cfg.vocab, (B, 40)).astype(np.int32)).cuda()
        out = dec.generate(ids, n_new=n_new)
        toks = [dec.prefill(ids)]
        for _ in range(n_new - 1):
            toks.append(dec.decode_step())
        assert torch.equal(out, torch.stack(toks, dim=1)), (B, n_new)
    no_device_error()


def test_decoder_int8():
    dev()
    cfg = SmallCfg()
    p = random_params(cfg, seed=5)
    dec = make(cfg, int8=True)
    upload(dec, p)
    ora = OracleDecoder(cfg, p, int8=True)
    ids = np.random.default_rng(2).integers(0, cfg.vocab, (2, 20)).astype(np.int32)
    nxt, logits = dec.prefill(torch.from_numpy(ids).cuda(), return_logits=True)
    ref = ora.forward(ids)
    assert_close(np_of(logits), ref, BF16_TOL, "int8 prefill")
    for _ in range(3):
        tok = np.argmax(ref, axis=1).astype(np.int32)
        nxt, logits = dec.decode_step(torch.from_numpy(tok).cuda(), return_logits=True)
        ref = ora.forward(tok[:, None])
        assert_close(np_of(logits), ref, BF16_TOL, "int8 decode")
    no_device_error()


@pytest.mark.parametrize("int8", [False, True])
def test_decoder_wide_split_k(int8):
    # d_model 1024 and ffn 2048 give the GEMVs enough K blocks to split K over a
    # cluster, so prefill (40 tokens) and decode (2 tokens) run the cluster exchange
    # together with the fused RMSNorm's sums of squares and the RoPE / KV-cache
    # epilogue; the small model's few K blocks never leave the single-CTA path
    dev()
    cfg = SmallCfg(d_model=1024, n_heads=16, n_kv_heads=4, ffn_hidden=2048, vocab=512)
    p = random_params(cfg, seed=6)
    dec = make(cfg, int8=int8)
    upload(dec, p)
    ora = OracleDecoder(cfg, p, int8=int8)
    ids = np.random.default_rng(11).integers(0, cfg.vocab, (2, 20)).astype(np.int32)
    nxt, logits = dec.prefill(torch.from_numpy(ids).cuda(), return_logits=True)
    ref = ora.forward(ids)
    assert_close(np_of(logits), ref, BF16_TOL, "prefill logits")
    for step in range(2):
        tok = np.argmax(ref, axis=1).astype(np.int32)
        nxt, logits = dec.decode_step(torch.from_numpy(tok).cuda(), return_logits=True)
        ref = ora.forward(tok[:, None])
        assert_close(np_of(logits), ref, BF16_TOL, f"decode step {step}")
    no_device_error()


def _oracle_with_cache(dec, cfg, p, B, length, int8):
    """Oracle decoder whose KV cache holds the executor's cache contents."""
    ora = OracleDecoder(cfg, p, int8=int8)
    ks, vs = [], []
    for l in range(cfg.n_layers):
        k, v = dec.read_kv(l, B, length)
        ks.append(k.float().cpu().numpy())
        vs.append(v.float().cpu().numpy())
    ora.k, ora.v, ora.len = np.stack(ks), np.stack(vs), length
    return ora


# The benchmarked model width (C4 / C5: d 2048, 32 / 8 heads x 64, SwiGLU 8192,
# vocab 32000) with 2 of its 16 layers, so every GEMV runs the benchmark's
# configuration: 16-CTA split-K clusters, fused RMSNorm, the RoPE / KV-cache
# epilogue, the 16-chunk argmax over 32000 logits.
C4_WIDTH = dict(n_layers=2, d_model=2048, n_heads=32, n_kv_heads=8, head_dim=64, ffn_hidden=8192, vocab=32000)


# chain: decode runs O, gate/up, down and the next layer's QKV of each layer as
# one persistent launch (opt-in, TB_DECODE_CHAIN=1); off: one GEMV launch per
# matrix (the default).
@pytest.mark.parametrize("chain", [True, False])
def test_decoder_c4_width_bf16(chain, monkeypatch):
    # prefill: 16 sequences x 16 tokens (256 rows: the tensor-core GEMM path and
    # prefill attention); then decode at batch 16 (the benchmark's decode GEMVs)
    dev()
    monkeypatch.setenv("TB_DECODE_CHAIN", "1" if chain else "0")
    cfg = SmallCfg(**C4_WIDTH)
    p = random_params(cfg, seed=12)
    dec = make(cfg, max_batch=16, max_seq=64)
    upload(dec, p)
    ora = OracleDecoder(cfg, p)
    ids = np.random.default_rng(13).integers(0, cfg.vocab, (16, 16)).astype(np.int32)
    nxt, logits = dec.prefill(torch.from_numpy(ids).cuda(), return_logits=True)
    ref = ora.forward(ids)
    assert_close(np_of(logits), ref, BF16_TOL, "prefill logits")
    check_tokens(nxt.cpu().numpy(), ref)
    for step in range(2):
        tok = np.argmax(ref, axis=1).astype(np.int32)
        nxt, logits = dec.decode_step(torch.from_numpy(tok).cuda(), return_logits=True)
        ref = ora.forward(tok[:, None])
        assert_close(np_of(logits), ref, BF16_TOL, f"decode step {step}")
        check_tokens(nxt.cpu().numpy(), ref)
    no_device_error()


def test_decoder_c5_width_int8_decode():
    # C5: int8 weights, decode-only batch 64 over a 2048-position cache of N(0, 1)
    # keys / values; the oracle is given the same cache contents
    dev()
    cfg = SmallCfg(**C4_WIDTH)
    p = random_params(cfg, seed=14)
    B, L = 64, 2048
    dec = make(cfg, int8=True, max_batch=B, max_seq=L + 8)
    upload(dec, p)
    tok = np.random.default_rng(15).integers(0, cfg.vocab, B).astype(np.int32)
    dec.fill_kv_random(torch.from_numpy(tok).cuda(), L, seed=16)
    ora = _oracle_with_cache(dec, cfg, p, B, L, int8=True)
    for step in range(2):
        nxt, logits = dec.decode_step(torch.from_numpy(tok).cuda(), return_logits=True)
        ref = ora.forward(tok[:, None])
        assert_close(np_of(logits), ref, BF16_TOL, f"int8 decode step {step}")
        check_tokens(nxt.cpu().numpy(), ref)
        tok = np.argmax(ref, axis=1).astype(np.int32)
    assert dec.seq_len() == L + 2
    no_device_error()


def test_decoder_fill_kv_random_decode_only():
    dev()
    cfg = SmallCfg()
    dec = make(cfg, int8=True, max_batch=8, max_seq=300)
    dec.init_random(seed=1)
    ids = torch.arange(8, dtype=torch.int32, device="cuda")
    dec.fill_kv_random(ids, 256, seed=3)
    a = dec.decode_step()
    b = dec.decode_step()
    assert a.shape == (8,) and int(a.max()) < cfg.vocab and int(b.min()) >= 0
    assert dec.seq_len() == 258
    no_device_error()


def test_decoder_rejects_bad_shapes():
    dev()
    from teenygrad_b200 import TeenyError
    cfg = SmallCfg()
    dec = make(cfg, max_seq=64)
    dec.init_random(0)
    with pytest.raises(TeenyError):
        dec.prefill(torch.zeros(5, 10, dtype=torch.int32, device="cuda"))   # B > max_batch
    with pytest.raises(TeenyError):
        dec.prefill(torch.zeros(1, 64, dtype=torch.int32, device="cuda"))   # S >= max_seq
