"""tb_argmax_noalloc_fwd: the argmax entry point that allocates no device memory.

Some callers cannot call cudaMalloc -- for instance a serving loop whose device
memory is owned by an external pool.  This entry point keeps its cross-block scratch in a static
device array instead.  The test calls it through the C ABI twice in a row (the
scratch keeps the previous call's contents, so the second call checks that it
starts clean) and compares each result with tb_argmax_fwd's, which must agree
exactly (argmax is bit-exact).  It is collected last so that a run stopping at
the first failure has already run every other test.
"""
import ctypes

import numpy as np
import pytest

import oracle
from gpu_util import bf16_round, dev, torch

pytestmark = pytest.mark.gpu

TB_F32, TB_BF16, TB_ERR_SHAPE, MAX_ROWS = 0, 1, 2, 4096


def _call(fn, ctx, dtype, x, out, M, N):
    return fn(ctx, ctypes.c_int(dtype), ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(out.data_ptr()),
              ctypes.c_int64(M), ctypes.c_int64(N))


def test_argmax_noalloc_matches_argmax_twice():
    dev()
    from teenygrad_b200 import _lib, ops
    lib = _lib.lib()
    ctx = ops.context()
    rng = np.random.default_rng(123)
    for call, (M, N, dtype) in enumerate([(64, 32000, TB_F32), (16, 50000, TB_F32), (7, 4100, TB_BF16)]):
        logits = rng.standard_normal((M, N)).astype(np.float32)
        logits[0, [5, 4000]] = 40.0          # tie across two blocks: lower index wins
        logits[1, :] = -np.inf
        logits[2, 17] = np.nan
        logits[3, :] = -1.0                  # maximum 0: -0.0 in the first block, +0.0 in a later one
        logits[3, 5] = -0.0
        logits[3, 4000] = 0.0
        logits[4, :] = -2.0                  # +0.0 first, -0.0 later
        logits[4, 9] = 0.0
        logits[4, 4090] = -0.0
        if dtype == TB_BF16:
            logits = bf16_round(logits)
        x = torch.from_numpy(logits).cuda()
        if dtype == TB_BF16:
            x = x.bfloat16()
        ref = torch.full((M,), -1, dtype=torch.int32, device="cuda")
        got = torch.full((M,), -2, dtype=torch.int32, device="cuda")
        _lib.check(ctx, _call(lib.tb_argmax_fwd, ctx, dtype, x, ref, M, N))
        _lib.check(ctx, _call(lib.tb_argmax_noalloc_fwd, ctx, dtype, x, got, M, N))
        torch.cuda.synchronize()
        assert torch.equal(got, ref), f"call {call}"
        np.testing.assert_array_equal(got.cpu().numpy(), oracle.argmax(logits), err_msg=f"call {call}")
        assert int(got[0]) == 5 and int(got[3]) == 5 and int(got[4]) == 9


def test_argmax_noalloc_rejects_too_many_rows():
    dev()
    from teenygrad_b200 import _lib, ops
    lib = _lib.lib()
    ctx = ops.context()
    x = torch.zeros(MAX_ROWS + 1, 8, device="cuda")
    out = torch.zeros(MAX_ROWS + 1, dtype=torch.int32, device="cuda")
    assert _call(lib.tb_argmax_noalloc_fwd, ctx, TB_F32, x, out, MAX_ROWS + 1, 8) == TB_ERR_SHAPE
    assert "static scratch" in lib.tb_last_error(ctx).decode()
