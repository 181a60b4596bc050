"""C1: fp32 pre-norm transformer block through the library vs the oracle (1e-4)."""
import numpy as np
import pytest

from gpu_util import F32_TOL, assert_close, dev, no_device_error, np_of, torch
from oracle.decoder import block_forward as oracle_block

pytestmark = pytest.mark.gpu


def test_block_c1_fp32():
    dev()
    from teenygrad_b200.block import block_forward, random_block_params
    p = random_block_params(seed=3)
    x = torch.randn(1, 128, 256, generator=torch.Generator().manual_seed(1)).cuda()
    y = block_forward(x, p, n_heads=4, eps=1e-6)
    ref = oracle_block(x.cpu().numpy(), {k: v.cpu().numpy() for k, v in p.items()}, 4, 1e-6)
    assert_close(np_of(y), ref, F32_TOL)
    no_device_error()
