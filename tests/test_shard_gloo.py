"""Row sharding with x broadcast and y all-gather, on world_size-2 gloo ranks (no GPU): every rank
must end with the full y equal to the single-process oracle result."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from l2domain_b200.shard import RowShard, ShardedGemvStep, unpad_gathered


@pytest.mark.parametrize("M,world", [(131072, 8), (10, 3), (7, 2), (1, 2), (4096, 4)])
def test_row_shards_cover_rows_once(M, world):
    shards = RowShard(M, world, 0).ranges()
    covered = []
    for s in shards:
        covered.extend(range(s.row0, s.row0 + s.rows))
        assert s.rows <= s.padded
    assert covered == list(range(M))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, M, N, out_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    import oracle as O

    shard = RowShard(M, world, rank)
    A = O.cfg_fill(M * N, 0, 0, O.NORMAL, 0.0, 0.02).reshape(M, N)[shard.row0: shard.row0 + shard.rows]
    x = torch.from_numpy(O.cfg_fill(N, 0, 1, O.NORMAL, 0.0, 1.0)) if rank == 0 else torch.zeros(N)
    y_local = torch.zeros(shard.padded)
    y_all = torch.zeros(shard.padded * world)

    def local():
        y_local[: shard.rows] = torch.from_numpy(O.gemv_seq(np.ascontiguousarray(A), x.numpy(), O.F32, shard.rows, N))

    ShardedGemvStep(shard, x, y_local, y_all, local)()
    out_q.put((rank, unpad_gathered(y_all, shard).numpy()))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("M,world", [(64, 2), (37, 2)])
def test_broadcast_gemv_allgather_two_ranks(M, world):
    import oracle as O

    N = 256
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, M, N, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    A = O.cfg_fill(M * N, 0, 0, O.NORMAL, 0.0, 0.02)
    x = O.cfg_fill(N, 0, 1, O.NORMAL, 0.0, 1.0)
    want = O.gemv_seq(A, x, O.F32, M, N)
    for r in range(world):
        assert np.array_equal(results[r], want)


def _dead_rank_worker(rank, world, port, q):
    """Rank 1 exits before the collective: rank 0's collective must fail, not hang."""
    from datetime import timedelta

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=5))
    if rank == 1:
        os._exit(0)
    x = torch.zeros(8)
    try:
        dist.broadcast(x, src=0)
        dist.all_reduce(x)
        q.put("no error")
    except Exception as e:  # noqa: BLE001
        q.put(type(e).__name__)


def test_dead_rank_surfaces_as_error():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_dead_rank_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert got != "no error"


def _exchange_worker(rank, world, port, q):
    """Each rank contributes a distinct blob; every rank must get all of them in rank order."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from l2domain_b200.shard import exchange_bytes

    blob = bytes((rank * 37 + k) % 256 for k in range(96))
    q.put((rank, exchange_bytes(blob)))
    dist.barrier()
    dist.destroy_process_group()


def test_handle_exchange_keeps_rank_order():
    world = 3
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_exchange_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    want = [bytes((r * 37 + k) % 256 for k in range(96)) for r in range(world)]
    for r in range(world):
        assert results[r] == want
