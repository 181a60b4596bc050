"""CPU checks of the oracle decoder composition (no GPU)."""
import numpy as np

from decoder_util import SmallCfg
from oracle.decoder import OracleDecoder, random_params


def test_kv_cache_consistency():
    cfg = SmallCfg(n_layers=1, vocab=256)
    p = random_params(cfg, seed=1)
    ids = np.random.default_rng(0).integers(0, cfg.vocab, (2, 9))
    full = OracleDecoder(cfg, p).forward(ids)
    inc = OracleDecoder(cfg, p)
    inc.forward(ids[:, :8])
    step = inc.forward(ids[:, 8:9])
    # same math, different rounding order only through bf16 of identical values
    np.testing.assert_allclose(step, full, atol=1e-4)


def test_int8_close_to_bf16():
    cfg = SmallCfg(n_layers=1, vocab=256)
    p = random_params(cfg, seed=2)
    ids = np.random.default_rng(1).integers(0, cfg.vocab, (1, 6))
    a = OracleDecoder(cfg, p).forward(ids)
    b = OracleDecoder(cfg, p, int8=True).forward(ids)
    assert np.abs(a - b).max() < 0.05 * max(1.0, np.abs(a).max())
