"""Row-sharded GEMV over the GPUs of one node (one process per GPU, torch.distributed).

The reference has no multi-GPU path; this is the sharded configuration of the build: GPU g owns
rows [row0(g), row0(g) + rows(g)) of A, x is broadcast from rank 0 and the y shards are
all-gathered so every rank ends with the whole y.  Two ways to run a step:

* :class:`PeerGemvStep` -- libl2d's l2d_gemv_sharded: the broadcast and the gather are folded into
  the GEMV launch over peer memory (CUDA IPC over NVLink); no collective library on the data path.
  torch.distributed only exchanges the IPC handles once, at set-up.
* :class:`ShardedGemvStep` -- NCCL broadcast, local GEMV, NCCL all-gather.  The same code runs on
  the gloo backend with CPU tensors, which is how the partitioning and gather order are tested
  without GPUs.

Shards are contiguous and as even as possible: the first M % world ranks get one extra row.
all_gather_into_tensor needs equal chunks, so y shards are padded to ceil(M / world) rows and the
padding is dropped after the gather.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable


@dataclass(frozen=True)
class RowShard:
    M: int
    world: int
    rank: int

    @property
    def rows(self) -> int:
        return self.M // self.world + (1 if self.rank < self.M % self.world else 0)

    @property
    def row0(self) -> int:
        base, extra = divmod(self.M, self.world)
        return self.rank * base + min(self.rank, extra)

    @property
    def padded(self) -> int:
        return -(-self.M // self.world)

    def ranges(self):
        return [RowShard(self.M, self.world, r) for r in range(self.world)]


def unpad_gathered(buf, shard: RowShard, elem_per_row: int = 1):
    """Drops the padding rows of a gathered [world * padded] buffer (any indexable 1-D tensor)."""
    if shard.M % shard.world == 0:
        return buf[: shard.M * elem_per_row]
    import torch

    parts = []
    for s in shard.ranges():
        lo = s.rank * shard.padded * elem_per_row
        parts.append(buf[lo: lo + s.rows * elem_per_row])
    return torch.cat(parts)


class ShardedGemvStep:
    """One sharded step: broadcast x from rank 0, run the local GEMV, all-gather y.

    ``local_gemv`` computes this rank's y shard into ``y_local`` (length ``padded`` rows; rows past
    ``shard.rows`` are padding); on the GPU it is the libl2d plan's call.  ``group`` is the
    torch.distributed process group (None = default)."""

    def __init__(self, shard: RowShard, x, y_local, y_gathered, local_gemv: Callable[[], None], group=None):
        self.shard, self.x, self.y_local, self.y_gathered = shard, x, y_local, y_gathered
        self.local_gemv, self.group = local_gemv, group

    def __call__(self):
        import torch.distributed as dist

        if self.shard.world > 1:
            dist.broadcast(self.x, src=0, group=self.group)
        self.local_gemv()
        if self.shard.world > 1:
            dist.all_gather_into_tensor(self.y_gathered, self.y_local, group=self.group)


def exchange_bytes(blob: bytes, group=None, device=None) -> list:
    """All-gathers one equally sized byte string per rank; returns them in rank order."""
    import torch
    import torch.distributed as dist

    world = dist.get_world_size(group)
    n = len(blob)
    mine = torch.tensor(list(blob), dtype=torch.uint8, device=device)
    out = torch.empty(world * n, dtype=torch.uint8, device=device)
    dist.all_gather_into_tensor(out, mine, group=group)
    raw = bytes(out.cpu().tolist())
    return [raw[i * n:(i + 1) * n] for i in range(world)]


class PeerGemvStep:
    """One sharded step through peer memory: ``l2d_gemv_sharded`` on this rank's plan.

    ``plan`` covers this rank's rows only (``shard.rows`` x N).  ``exchange`` maps this rank's
    handle blob to all ranks' blobs in rank order (:func:`exchange_bytes` under torch.distributed).
    Rank 0 writes a step's x into ``x(parity)`` with ``parity = next_parity()`` before the call;
    after the call (stream-ordered) ``y(parity)`` holds all M rows on every rank.
    """

    def __init__(self, shard: RowShard, plan, N: int, dtype_in: int, dtype_out: int, device: int,
                 exchange: Callable[[bytes], list], timeout_ms: int = 2000):
        import l2domain_b200 as L

        self.shard = shard
        self.plan = plan
        self.peer = L.PeerShard(device, shard.rank, shard.world, shard.M, shard.row0, shard.rows, N, dtype_in,
                                dtype_out, timeout_ms)
        self.peer.connect(exchange(self.peer.handle()))

    def next_parity(self) -> int:
        return self.peer.next_parity()

    def x(self, parity: int):
        return self.peer.x_tensor(parity)

    def y(self, parity: int):
        return self.peer.y_tensor(parity)

    def __call__(self, mode: int = 1, stream=None) -> int:
        return self.peer.step(self.plan, mode, stream)

    def status(self) -> int:
        return self.peer.status()

    def close(self) -> None:
        self.peer.close()
