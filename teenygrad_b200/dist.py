"""Batch-sharded multi-GPU helpers: one process per GPU, outputs all-gathered.

The hot path shards by independent sequences / images / heads; the only
collective is the all-gather of the final outputs.  torch.distributed is the
bootstrap (rank / world size and the exchange of NCCL's unique id); the
all-gather itself runs through the library's communicator (tb_comm_*).
"""
from __future__ import annotations

import ctypes

import torch

from ._lib import TeenyError, check, lib
from .ops import context


def shard(n: int, world: int, rank: int) -> tuple[int, int]:
    """(start, count) of rank's contiguous share of n units; the first n % world
    ranks take one extra unit."""
    if world < 1 or not 0 <= rank < world:
        raise TeenyError(1, f"shard: rank {rank} of {world}")
    base, extra = divmod(n, world)
    start = rank * base + min(rank, extra)
    return start, base + (1 if rank < extra else 0)


def exchange_unique_id(get_id, broadcast, rank: int) -> bytes:
    """Rank 0 creates the NCCL id with get_id(); broadcast(tensor, src=0) shares
    it (a torch.distributed broadcast on any backend)."""
    n = lib().tb_comm_unique_id_bytes()
    buf = torch.zeros(n, dtype=torch.uint8)
    if rank == 0:
        buf.copy_(torch.frombuffer(bytearray(get_id()), dtype=torch.uint8))
    broadcast(buf, src=0)
    return bytes(buf.tolist())


def nccl_unique_id() -> bytes:
    n = lib().tb_comm_unique_id_bytes()
    out = ctypes.create_string_buffer(n)
    st = lib().tb_comm_get_unique_id(out)
    if st != 0:
        raise TeenyError(st, "tb_comm_get_unique_id failed")
    return out.raw


class Comm:
    """The library's NCCL communicator for this process's GPU."""

    def __init__(self, rank: int, world: int, timeout_ms: int = 60000, device: int | None = None):
        import torch.distributed as dist
        self.rank, self.world = rank, world
        self.device = torch.cuda.current_device() if device is None else device
        self.ctx = context(self.device)
        uid = exchange_unique_id(nccl_unique_id, lambda t, src: self._bcast(dist, t, src), rank)
        check(self.ctx, lib().tb_comm_init(self.ctx, ctypes.c_char_p(uid), ctypes.c_int(world), ctypes.c_int(rank),
                                          ctypes.c_int(timeout_ms)))

    @staticmethod
    def _bcast(dist, t, src):
        if dist.get_backend() == "nccl":
            g = t.cuda()
            dist.broadcast(g, src=src)
            t.copy_(g.cpu())
        else:
            dist.broadcast(t, src=src)

    def all_gather(self, local: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        local = local.contiguous()
        if out is None:
            out = torch.empty((self.world * local.shape[0],) + tuple(local.shape[1:]), dtype=local.dtype,
                              device=local.device)
        ctx = context(self.device)
        check(ctx, lib().tb_comm_allgather(ctx, ctypes.c_void_p(local.data_ptr()), ctypes.c_void_p(out.data_ptr()),
                                           ctypes.c_size_t(local.numel() * local.element_size())))
        return out

    def close(self):
        lib().tb_comm_destroy(self.ctx)
