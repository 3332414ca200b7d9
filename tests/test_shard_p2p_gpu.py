"""Row-sharded GEMV over peer memory (l2d_gemv_sharded) on the GPU.

* one rank (world 1): the sharded step must give bit-for-bit the planned GEMV's y;
* bounded waits: a world-2 shard whose peer never runs (its flags are never set) must return with
  both timeout bits set and leave the context usable -- the failure is made by a flag nothing
  sets, never by a fault;
* two GPUs (skipped with fewer): two processes exchange IPC handles over NCCL and run three
  steps; every rank's gathered y must equal the all-gather of the planned GEMV's shards exactly.
  The row split is ragged (5003 rows), so a shard starts at a byte offset that is not 16-aligned;
  with one row in all, rank 1 owns none and still takes part in every step.
"""
import os
import socket

import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import l2domain_b200 as L  # noqa: E402
from l2domain_b200.shard import RowShard  # noqa: E402

PAGE = 2 * 1024 * 1024


def aligned(nbytes, device):
    region = (nbytes + PAGE - 1) // PAGE * PAGE
    raw = torch.empty(region + PAGE, dtype=torch.uint8, device=device)
    off = (-raw.data_ptr()) % PAGE
    return raw, raw[off: off + nbytes]


def need_gpu(n=1):
    if not torch.cuda.is_available() or torch.cuda.device_count() < n:
        pytest.skip(f"needs {n} GPU(s)")


def test_single_rank_sharded_step_equals_planned_gemv():
    need_gpu()
    torch.cuda.set_device(0)
    M, N = 3001, 4096
    keep, A = aligned(M * N * 2, "cuda")
    L.fill_cfg(A, L.F16, M * N, 5, 0, 1, 0.0, 0.02)
    plan = L.GemvPlan(A, M, N, L.F16, L.F16)
    sh = L.PeerShard(0, 0, 1, M, 0, M, N, L.F16, L.F16)
    sh.connect([sh.handle()])
    for step in range(3):
        par = sh.next_parity()
        xb = sh.x_tensor(par)
        L.fill_cfg(xb, L.F16, N, 100 + step, 1, 1, 0.0, 1.0)
        y_ref = torch.empty(M * 2, dtype=torch.uint8, device="cuda")
        plan.gemv(A, xb, y_ref, L.MODE_AWARE)
        assert sh.step(plan, L.MODE_AWARE) == par
        torch.cuda.synchronize()
        assert torch.equal(sh.y_tensor(par), y_ref), f"step {step}"
    assert sh.status() == 0
    sh.close()
    plan.close()


def test_missing_peer_times_out_with_status_bits():
    need_gpu()
    torch.cuda.set_device(0)
    M, N = 2048, 1024
    row0, rows = 1024, 1024
    keep, A = aligned(rows * N * 2, "cuda")
    L.fill_cfg(A, L.F16, rows * N, 5, 0, 1, 0.0, 0.02, first=row0 * N)
    plan = L.GemvPlan(A, rows, N, L.F16, L.F16)
    # Both ranks' shard objects live in this process; only rank 1 ever steps, so rank 0 never pushes x
    # and never publishes its rows: rank 1's two waits must run out after 50 ms each.
    s0 = L.PeerShard(0, 0, 2, M, 0, 1024, N, L.F16, L.F16, timeout_ms=50)
    s1 = L.PeerShard(0, 1, 2, M, row0, rows, N, L.F16, L.F16, timeout_ms=50)
    blobs = [s0.handle(), s1.handle()]
    s0.connect(blobs)
    s1.connect(blobs)
    s1.step(plan, L.MODE_AWARE)
    assert s1.status() == 3
    # The context is still usable: a plain GEMV after the timeouts is correct.
    x = torch.empty(N * 2, dtype=torch.uint8, device="cuda")
    L.fill_cfg(x, L.F16, N, 7, 1, 1, 0.0, 1.0)
    y = torch.empty(rows * 2, dtype=torch.uint8, device="cuda")
    plan.gemv(A, x, y, L.MODE_AWARE)
    torch.cuda.synchronize()
    ref = (A.view(torch.float16).view(rows, N).double() @ x.view(torch.float16).double())
    got = y.view(torch.float16).double()
    assert float((got - ref).norm() / ref.norm()) <= 2e-3
    s1.close()
    s0.close()
    plan.close()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _two_gpu_worker(rank, world, port, M, N, q):
    from datetime import timedelta

    import torch.distributed as dist

    from l2domain_b200.shard import PeerGemvStep, exchange_bytes

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
    try:
        shard = RowShard(M, world, rank)
        keep, A = aligned(max(shard.rows, 1) * N * 2, dev)
        L.fill_cfg(A, L.F16, shard.rows * N, 9, 0, 1, 0.0, 0.02, first=shard.row0 * N)
        plan = L.GemvPlan(A, shard.rows, N, L.F16, L.F16, device=rank)
        step = PeerGemvStep(shard, plan, N, L.F16, L.F16, rank, lambda b: exchange_bytes(b, device=dev))
        x = torch.empty(N * 2, dtype=torch.uint8, device=dev)
        y_loc = torch.zeros(shard.padded * 2, dtype=torch.uint8, device=dev)
        y_all = torch.empty(shard.padded * world * 2, dtype=torch.uint8, device=dev)
        bad = []
        for k in range(3):
            L.fill_cfg(x, L.F16, N, 200 + k, 1, 1, 0.0, 1.0)
            plan.gemv(A, x, y_loc, L.MODE_AWARE)
            dist.all_gather_into_tensor(y_all, y_loc)
            want = torch.cat([y_all[s.rank * shard.padded * 2: (s.rank * shard.padded + s.rows) * 2]
                              for s in shard.ranges()])
            par = step.next_parity()
            if rank == 0:
                step.x(par).copy_(x)
            step(L.MODE_AWARE)
            torch.cuda.synchronize()
            if not torch.equal(step.y(par), want):
                bad.append(k)
        st = step.status()
        dist.barrier(device_ids=[rank])
        step.close()
        plan.close()
        q.put((rank, bad, st))
    finally:
        dist.destroy_process_group()


def _cfg5_worker(rank, world, port, M, N, rows_sample, q):
    from datetime import timedelta

    import torch.distributed as dist

    from l2domain_b200.shard import PeerGemvStep, exchange_bytes

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120), device_id=dev)
    try:
        shard = RowShard(M, world, rank)
        keep, A = aligned(shard.rows * N * 2, dev)
        L.fill_cfg(A, L.F16, shard.rows * N, 0, 0, 1, 0.0, 0.02, first=shard.row0 * N)
        plan = L.GemvPlan(A, shard.rows, N, L.F16, L.F16, device=rank)
        step = PeerGemvStep(shard, plan, N, L.F16, L.F16, rank, lambda b: exchange_bytes(b, device=dev))
        out = {}
        for mode in (L.MODE_AWARE, L.MODE_STREAM):
            for k in range(2):
                par = step.next_parity()
                if rank == 0:
                    L.fill_cfg(step.x(par), L.F16, N, 0, 1, 1, 0.0, 1.0)
                step(mode)
                torch.cuda.synchronize()
            out[mode] = step.y(par).view(torch.int16)[torch.as_tensor(rows_sample, device=dev)].cpu().numpy()
        st = step.status()
        dist.barrier(device_ids=[rank])
        step.close()
        plan.close()
        q.put((rank, out, st))
    finally:
        dist.destroy_process_group()


def test_all_gpus_cfg5_gathered_y_matches_oracle():
    """Config 5 at full size (fp16 A 131072 x 16384, 4 GiB) row-sharded over every visible GPU,
    two steps per mode with x from rank 0: on every rank, the gathered y of sampled rows of every
    rank's shard (its first, middle and last 64 rows) is checked against the CPU oracle (relative
    L2 <= 2e-3 of the fp64 result of the same rounded inputs), and all ranks hold the same bits."""
    need_gpu(2)
    import numpy as np
    import torch.multiprocessing as mp

    import oracle as O

    M, N, world = 131072, 16384, torch.cuda.device_count()
    shards = [RowShard(M, world, r) for r in range(world)]
    rows = np.unique(np.concatenate([np.r_[s.row0: s.row0 + 64, s.row0 + s.rows // 2 - 32: s.row0 + s.rows // 2 + 32,
                                           s.row0 + s.rows - 64: s.row0 + s.rows] for s in shards]))
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_cfg5_worker, args=(r, world, port, M, N, rows, q)) for r in range(world)]
    for p in procs:
        p.start()
    x_h = O.round_to(O.cfg_fill(N, 0, 1, O.NORMAL, 0.0, 1.0), O.F16)
    runs = np.split(rows, np.where(np.diff(rows) != 1)[0] + 1)
    y64 = np.concatenate([O.gemv_f64(O.round_to(O.cfg_fill(len(r) * N, 0, 0, O.NORMAL, 0.0, 0.02,
                                                           first=int(r[0]) * N, threads=0), O.F16),
                                     x_h, O.F16, len(r), N) for r in runs])
    ref = O.round_out(y64, O.F16).astype(np.float64)
    results = dict((r, (o, s)) for r, o, s in (q.get(timeout=600) for _ in range(world)))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for r in range(world):
        outs, st = results[r]
        assert st == 0, f"rank {r} timeout bits {st}"
        for mode, y in outs.items():
            got = O.widen(y.view(np.uint16), O.F16)
            err = O.rel_l2(ref, got)
            assert err <= 2e-3, f"rank {r} mode {mode}: rel L2 {err:.3g}"
            assert np.array_equal(y, results[0][0][mode]), f"rank {r} mode {mode}: differs from rank 0"


@pytest.mark.parametrize("M", [5003, 1])
def test_two_gpus_gather_equals_nccl_allgather(M):
    """M = 1 leaves rank 1 without rows: it still takes part in every step."""
    need_gpu(2)
    import torch.multiprocessing as mp

    N, world = 8192, 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_two_gpu_worker, args=(r, world, port, M, N, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict((r, (b, s)) for r, b, s in (q.get(timeout=300) for _ in range(world)))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for r in range(world):
        bad, st = results[r]
        assert st == 0, f"rank {r} timeout bits {st}"
        assert not bad, f"rank {r}: gathered y differs at steps {bad}"
