"""Helpers for the GPU parity tests (CUDA path vs the CPU oracle)."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

import oracle  # noqa: E402

BF16_TOL = 2e-2   # bf16 tensor-core paths, f32 accumulate
F32_TOL = 1e-4    # fp32 paths


def dev():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    return torch.device("cuda", 0)


def to_gpu(a, dtype=torch.float32):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev()).to(dtype).contiguous()


def bf16_round(a):
    return oracle.round_bf16(np.asarray(a, np.float32))


def np_of(t):
    return t.detach().float().cpu().numpy()


def assert_close(got, ref, tol, what=""):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    assert got.shape == ref.shape, (got.shape, ref.shape)
    assert np.all(np.isfinite(got)), f"{what}: non-finite output"
    scale = max(1.0, float(np.abs(ref).max())) if ref.size else 1.0
    err = float(np.abs(got - ref).max()) if ref.size else 0.0
    assert err <= tol * scale, f"{what}: max abs err {err:.3e} > {tol} * {scale:.3e}"
    return err


def rng(seed=0):
    return np.random.default_rng(seed)


def no_device_error():
    from teenygrad_b200 import ops
    code = ops.device_error(clear=True)
    assert code == 0, f"device error word {code:#x}"
