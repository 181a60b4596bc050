"""Host-side multi-rank logic on CPU (gloo, world size 2): sharding, the NCCL
unique-id exchange pattern, output gathering order, and a failing rank."""
import os
import socket
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from teenygrad_b200.dist import exchange_unique_id, shard


def test_shard_covers_everything():
    for n in (0, 1, 7, 16, 64, 256):
        for world in (1, 2, 3, 4, 8):
            got = [shard(n, world, r) for r in range(world)]
            assert sum(c for _, c in got) == n
            pos = 0
            for s, c in got:
                assert s == pos
                pos += c
            assert max(c for _, c in got) - min(c for _, c in got) <= 1


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q, mode):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=10))
    try:
        if mode == "ok":
            uid = exchange_unique_id(lambda: bytes(range(128)), dist.broadcast, rank)
            # each rank "generates" its shard of a global batch; all_gather restores global order
            start, cnt = shard(16, world, rank)
            local = torch.arange(start, start + cnt, dtype=torch.int32).repeat_interleave(3).view(cnt, 3)
            outs = [torch.empty_like(local) for _ in range(world)]
            dist.all_gather(outs, local)
            full = torch.cat(outs)
            q.put((rank, uid == bytes(range(128)), full[:, 0].tolist()))
        else:
            if rank == 1:
                raise RuntimeError("rank 1 fails before the collective")
            try:
                dist.all_gather([torch.zeros(1) for _ in range(world)], torch.ones(1))
                q.put((rank, "no error"))
            except Exception as e:   # the peer is gone: the collective errors out, no hang
                q.put((rank, type(e).__name__))
    except RuntimeError:
        q.put((rank, "raised"))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def _run(mode, world=2):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, world, port, q, mode)) for r in range(world)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(60)
    alive = [p for p in ps if p.is_alive()]
    for p in alive:
        p.kill()
    assert not alive, "a rank hung"
    return sorted([q.get(timeout=5) for _ in range(world)], key=lambda t: t[0])


def test_gloo_unique_id_exchange_and_gather():
    res = _run("ok")
    for rank, uid_ok, ids in res:
        assert uid_ok
        assert ids == list(range(16))


def test_gloo_failed_rank_is_detected():
    res = _run("fail")
    assert res[1] == (1, "raised")
    assert res[0][1] != "no error"
