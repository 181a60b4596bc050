"""Failure detection on the GPU, in the forms that fault, trap or hang no GPU.

* A device-side bounded wait that runs out: tb_selftest_bounded_wait waits on an
  mbarrier nothing arrives on (the same mbar_wait code every kernel uses), with
  a short limit in one CTA; the other CTA, on the normal multi-second limit,
  must return early once the first has flagged the error word.  The host reads
  the error word and the context keeps working.
* A missing peer: rank 0 of a 2-rank communicator calls tb_comm_init and rank 1
  never does.  The non-blocking NCCL init makes no progress, the library's
  bounded host wait runs out and aborts the communicator (TB_ERR_NCCL).  Only
  one GPU is touched (rank 1 does not exist); NVLS is off.
"""
import ctypes
import os
import subprocess
import sys
import textwrap
import time

import numpy as np
import pytest

from gpu_util import dev, torch

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
TB_ERR_NCCL, DEV_ERR_TIMEOUT_MISC = 7, 1 << 3


def test_bounded_wait_runs_out_and_context_survives():
    dev()
    from teenygrad_b200 import _lib, ops
    lib = _lib.lib()
    ctx = ops.context()
    assert ops.device_error(clear=True) == 0
    elapsed = torch.zeros(2, dtype=torch.int64, device="cuda")
    t0 = time.perf_counter()
    _lib.check(ctx, lib.tb_selftest_bounded_wait(ctx, ctypes.c_int(2000), ctypes.c_void_p(elapsed.data_ptr())))
    code = ops.device_error(clear=True)          # synchronises the stream
    wall = time.perf_counter() - t0
    e = elapsed.cpu().numpy()
    assert code & DEV_ERR_TIMEOUT_MISC, f"error word {code:#x}"
    assert 2_000_000 <= e[0] < 1_000_000_000, e     # the short wait gave up after its 2 ms limit
    assert 0 < e[1] < 1_000_000_000, e               # the long wait returned early (limit is seconds)
    assert wall < 3.0
    # the context still runs kernels, and the error word is clear again
    x = torch.randn(4, 256, device="cuda")
    y = ops.rms_norm(x, torch.ones(256, device="cuda"), eps=1e-6)
    torch.cuda.synchronize()
    ref = x / torch.sqrt((x * x).mean(-1, keepdim=True) + 1e-6)
    assert torch.allclose(y, ref, atol=1e-5)
    assert ops.device_error(clear=True) == 0


_MISSING_PEER = textwrap.dedent("""
    import ctypes, sys, time
    sys.path.insert(0, {root!r})
    import torch
    from teenygrad_b200 import _lib, ops
    lib = _lib.lib()
    ctx = ops.context(0)
    n = lib.tb_comm_unique_id_bytes()
    uid = ctypes.create_string_buffer(n)
    assert lib.tb_comm_get_unique_id(uid) == 0
    t0 = time.perf_counter()
    st = lib.tb_comm_init(ctx, uid, ctypes.c_int(2), ctypes.c_int(0), ctypes.c_int(3000))
    dt = time.perf_counter() - t0
    print("STATUS", st, "%.2f" % dt, lib.tb_last_error(ctx).decode(), flush=True)
    # the context stays usable after the abort
    x = torch.ones(2, 64, device="cuda")
    y = ops.rms_norm(x, torch.ones(64, device="cuda"))
    torch.cuda.synchronize()
    print("AFTER", float(y.sum()), flush=True)
""")


def test_comm_init_without_peer_times_out():
    dev()
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", CUDA_VISIBLE_DEVICES=os.environ.get("CUDA_VISIBLE_DEVICES", "0").split(",")[0])
    r = subprocess.run(["timeout", "-k", "10", "120", sys.executable, "-c", _MISSING_PEER.format(root=ROOT)],
                       capture_output=True, text=True, env=env)
    out = r.stdout
    assert r.returncode == 0, r.stdout + r.stderr
    line = [l for l in out.splitlines() if l.startswith("STATUS")][0].split()
    status, secs = int(line[1]), float(line[2])
    assert status == TB_ERR_NCCL, out
    assert 2.5 <= secs < 60, out
    assert "aborted" in out
    assert "AFTER 128.0" in out
