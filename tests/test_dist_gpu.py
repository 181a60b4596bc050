"""Multi-GPU: the library's NCCL all-gather across ranks (one process per GPU).
Skipped unless at least two GPUs are visible."""
import os
import socket
from datetime import timedelta

import pytest

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    from teenygrad_b200.dist import Comm, shard
    comm = Comm(rank, world, timeout_ms=30000, device=rank)
    start, cnt = shard(8 * world, world, rank)
    local = torch.arange(start, start + cnt, dtype=torch.int32, device="cuda").repeat_interleave(5).view(cnt, 5)
    full = comm.all_gather(local)
    torch.cuda.synchronize()
    q.put((rank, full[:, 0].cpu().tolist()))
    comm.close()
    dist.destroy_process_group()


def test_allgather_two_gpus():
    torch = pytest.importorskip("torch")
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(120)
    assert all(not p.is_alive() for p in ps), "a rank hung"
    res = sorted([q.get(timeout=5) for _ in range(2)])
    for _, ids in res:
        assert ids == list(range(16))
