"""GPU parity of the granule-ring (TMA bulk copy) kernels, plans made with L2D_PLAN_TMA.

Same bars as the register kernels: fp32 relative L2 <= 1e-5 and fp16/bf16 <= 2e-3 against the fp64
oracle (of the same rounded inputs, rounded to the output type); the exact-integer inputs
bit-exact.  The ring kernels claim rows from pools, so the tests also pin what must not depend on
who claimed what: AWARE and SWAPPED bit-identical on every split-pool row (the same two partials,
added commutatively), rows taken whole bit-identical with STREAM (one warp, granules in order),
repeated calls bit-identical whatever ran in between (the exchange words empty themselves, the pool
counters reset).  Batched calls run the ring kernels too when every problem's rows sit on 4 KiB
granules (x then comes through L1 per problem); shapes the ring kernels cannot take (rows or
problem strides off the 4 KiB granules) run the register kernels.
"""
import json
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import l2domain_b200 as L  # noqa: E402
import oracle as O  # noqa: E402

GOLD = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "reference_pins.json")))
TOL = {L.F32: 1e-5, L.F16: 2e-3, L.BF16: 2e-3}
ALL_MODES = [L.MODE_OBLIVIOUS, L.MODE_AWARE, L.MODE_SWAPPED, L.MODE_STREAM]
PAGE = 2 * 1024 * 1024


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    torch.cuda.set_device(0)
    return torch.device("cuda", 0)


def to_dev(a):
    if a.dtype == np.uint16:
        a = a.view(np.int16)
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def inputs(M, N, dtype, batch=1, kind="cfg"):
    if kind == "int":
        A32 = O.ref_fill(batch * M * N, 4242, 0, integer_mode=True)
        x32 = O.ref_fill(batch * N, 4242, 1, integer_mode=True)
    else:
        A32 = O.cfg_fill(batch * M * N, 0, 0, O.NORMAL, 0.0, 0.02)
        x32 = O.cfg_fill(batch * N, 0, 1, O.NORMAL, 0.0, 1.0)
    return O.round_to(A32, dtype), O.round_to(x32, dtype)


def run(A_h, x_h, M, N, dtype, dtype_out, modes, batch=1, tma=True, placement=None):
    nbytes = A_h.nbytes
    raw = torch.empty(nbytes + PAGE, dtype=torch.uint8, device="cuda")
    off = (-raw.data_ptr()) % PAGE
    A = raw[off: off + nbytes]
    A.copy_(to_dev(A_h).view(torch.uint8).reshape(-1))
    x = to_dev(x_h)
    plan = L.GemvPlan(A, M, N, dtype, dtype_out, batch=batch, tma=tma, placement=placement)
    outs = {}
    for mode in modes:
        if dtype_out == L.F32:
            y = torch.full((batch * M,), float("nan"), dtype=torch.float32, device="cuda")
        else:
            y = torch.full((batch * M,), -1, dtype=torch.int16, device="cuda")
        plan.gemv(A, x, y, mode)
        torch.cuda.synchronize()
        yh = y.cpu().numpy()
        outs[mode] = yh if dtype_out == L.F32 else O.widen(yh.view(np.uint16), dtype_out)
    stats = plan.stats()
    plan.close()
    return outs, stats


def oracle(A, x, dtype, M, N, batch, dtype_out):
    ys = [O.gemv_f64(A[b * M * N:(b + 1) * M * N], x[b * N:(b + 1) * N], dtype, M, N, N) for b in range(batch)]
    y = np.concatenate(ys)
    return O.round_out(y, dtype_out) if dtype_out != L.F32 else y


@pytest.mark.parametrize("M,N,dtype,dtype_out,batch", [
    (3000, 4096, L.F16, L.F16, 1),     # 8 KiB rows: 2 granules
    (2049, 8192, L.BF16, L.BF16, 1),   # 16 KiB rows
    (1500, 2048, L.F32, L.F32, 1),     # 8 KiB fp32 rows
    (513, 16384, L.F16, L.F32, 1),     # 32 KiB rows, fp32 out
    (7, 2048, L.BF16, L.F32, 1),       # fewer rows than warps
    (20000, 1024, L.F32, L.F32, 1),    # 4 KiB rows: one granule, so every row is whole for one group
])
def test_ring_kernels_match_oracle(dev, M, N, dtype, dtype_out, batch):
    A, x = inputs(M, N, dtype, batch)
    outs, stats = run(A, x, M, N, dtype, dtype_out, ALL_MODES, batch)
    assert stats["tma"] == 2 and stats["device_errors"] == 0
    ref = oracle(A, x, dtype, M, N, batch, dtype_out)
    for m in ALL_MODES:
        err = O.rel_l2(ref.astype(np.float64), outs[m])
        assert err <= TOL[dtype], f"mode {m}: rel L2 {err:.3g}"


def test_ring_kernels_integer_kat_bit_exact(dev):
    g = GOLD["integer_kat"]
    M, N = g["M"], g["K"]
    A, x = inputs(M, N, L.F32, kind="int")
    outs, stats = run(A, x, M, N, L.F32, L.F32, ALL_MODES)
    assert stats["tma"] == 2
    want = np.array(g["y"], np.float32)
    for m in ALL_MODES:
        assert np.array_equal(outs[m], want), f"mode {m}"


def test_ring_kernels_aware_swapped_identical_and_deterministic(dev):
    M, N = 1024, 8192
    A, x = inputs(M, N, L.F16)
    outs, stats = run(A, x, M, N, L.F16, L.F32, [L.MODE_AWARE, L.MODE_SWAPPED, L.MODE_STREAM], placement="granules")
    assert stats["placement"] == 0
    whole = stats["ring_whole_rows"]
    assert 0 < whole < M // 4 and stats["ring_chunk_rows"] >= 1
    pool = M - whole
    assert np.array_equal(outs[L.MODE_AWARE][:pool], outs[L.MODE_SWAPPED][:pool])
    # Whole rows (one warp, every granule in order) are STREAM's arithmetic exactly.
    assert np.array_equal(outs[L.MODE_AWARE][pool:], outs[L.MODE_STREAM][pool:])
    outs2, _ = run(A, x, M, N, L.F16, L.F32, [L.MODE_AWARE], placement="granules")
    assert np.array_equal(outs[L.MODE_AWARE], outs2[L.MODE_AWARE])


def test_ring_calls_repeat_bit_identical_across_modes(dev):
    """Six calls on one plan, modes interleaved, launched back to back (each launch may overlap the
    previous call's tail): every AWARE call gives the same bits, so each call leaves the exchange
    words empty and the pool counters at zero for the next, and no call reads state early."""
    M, N = 3000, 4096
    A_h, x_h = inputs(M, N, L.BF16)
    nbytes = A_h.nbytes
    raw = torch.empty(nbytes + PAGE, dtype=torch.uint8, device="cuda")
    off = (-raw.data_ptr()) % PAGE
    A = raw[off: off + nbytes]
    A.copy_(to_dev(A_h).view(torch.uint8).reshape(-1))
    x = to_dev(x_h)
    plan = L.GemvPlan(A, M, N, L.BF16, L.F32, tma=True)
    modes = [L.MODE_AWARE, L.MODE_OBLIVIOUS, L.MODE_AWARE, L.MODE_STREAM, L.MODE_SWAPPED, L.MODE_AWARE]
    outs = [torch.full((M,), float("nan"), dtype=torch.float32, device="cuda") for _ in modes]
    torch.cuda.synchronize()
    for mode, y in zip(modes, outs):
        plan.gemv(A, x, y, mode)
    torch.cuda.synchronize()
    ys = [y for mode, y in zip(modes, outs) if mode == L.MODE_AWARE]
    stats = plan.stats()
    plan.close()
    assert stats["calls"] == 6 and stats["device_errors"] == 0 and stats["fallback_slots"] == 0
    for y in ys[1:]:
        assert torch.equal(y, ys[0])
    ref = oracle(A_h, x_h, L.BF16, M, N, 1, L.F32)
    assert O.rel_l2(ref.astype(np.float64), ys[0].cpu().numpy()) <= TOL[L.BF16]


def test_ring_kernels_agree_with_register_kernels(dev):
    M, N = 4096, 8192
    A, x = inputs(M, N, L.BF16)
    ring, s1 = run(A, x, M, N, L.BF16, L.F32, [L.MODE_AWARE], tma=True)
    reg, s0 = run(A, x, M, N, L.BF16, L.F32, [L.MODE_AWARE], tma=False)
    assert s1["tma"] == 2 and s0["tma"] == 0
    a, b = ring[L.MODE_AWARE].astype(np.float64), reg[L.MODE_AWARE].astype(np.float64)
    assert np.linalg.norm(a - b) / np.linalg.norm(b) <= 1e-5


@pytest.mark.parametrize("M,N,dtype,dtype_out,batch,pad_a,pad_x,pad_y", [
    (300, 4096, L.F16, L.F16, 3, 0, 0, 0),          # contiguous batch, 8 KiB rows
    (1000, 8192, L.BF16, L.BF16, 5, 4096, 24, 7),   # problem stride padded by one granule, x and y padded
    (64, 2048, L.F32, L.F32, 9, 8192, 4, 1),        # few rows per problem: chunks straddle problems
    (5, 16384, L.F16, L.F32, 40, 0, 8, 3),          # 32 KiB rows, more problems than rows per problem
])
def test_batched_ring_kernels_match_oracle(dev, M, N, dtype, dtype_out, batch, pad_a, pad_x, pad_y):
    """Batched calls on the granule-ring kernels (every problem's rows on 4 KiB granules): x of each
    problem is read through L1, y of problem b lands at b * stride_y."""
    eb = L.ELEM_BYTES[dtype]
    sa, sx, sy = M * N + pad_a // eb, N + pad_x, M + pad_y
    n_a, n_x = (batch - 1) * sa + M * N, (batch - 1) * sx + N
    A_h = O.round_to(O.cfg_fill(n_a, 1, 0, O.NORMAL, 0.0, 0.02), dtype)
    x_h = O.round_to(O.cfg_fill(n_x, 1, 1, O.NORMAL, 0.0, 1.0), dtype)
    raw = torch.empty(A_h.nbytes + PAGE, dtype=torch.uint8, device="cuda")
    off = (-raw.data_ptr()) % PAGE
    A = raw[off: off + A_h.nbytes]
    A.copy_(to_dev(A_h).view(torch.uint8).reshape(-1))
    x = to_dev(x_h)
    plan = L.GemvPlan(A, M, N, dtype, dtype_out, batch=batch, stride_a=sa, stride_x=sx, stride_y=sy, tma=True)
    st = plan.stats()
    assert st["tma"] == 2 and st["ring_modes"] == 0b1111
    y64 = np.concatenate([O.gemv_f64(A_h[b * sa: b * sa + M * N], x_h[b * sx: b * sx + N], dtype, M, N)
                          for b in range(batch)])
    ref = (O.round_out(y64, dtype_out) if dtype_out != L.F32 else y64).astype(np.float64)
    rows = np.concatenate([np.arange(b * sy, b * sy + M) for b in range(batch)])
    n_y = (batch - 1) * sy + M
    for m in ALL_MODES:
        if dtype_out == L.F32:
            y = torch.full((n_y,), float("nan"), dtype=torch.float32, device="cuda")
        else:
            y = torch.full((n_y,), -1, dtype=torch.int16, device="cuda")
        plan.gemv(A, x, y, m)
        torch.cuda.synchronize()
        yh = y.cpu().numpy()
        got = yh if dtype_out == L.F32 else O.widen(yh.view(np.uint16), dtype_out)
        err = O.rel_l2(ref, got[rows])
        assert err <= TOL[dtype], f"mode {m}: rel L2 {err:.3g}"
        pad = np.setdiff1d(np.arange(n_y), rows)  # rows between problems are never written
        if dtype_out == L.F32:
            assert np.all(np.isnan(yh[pad]))
        else:
            assert np.all(yh[pad] == -1)
    st = plan.stats()
    assert st["device_errors"] == 0
    plan.close()


def test_batched_off_granule_stride_runs_register_kernels(dev):
    M, N, batch = 300, 4096, 3  # problem stride not a multiple of 4 KiB
    sa = M * N + 8
    A_h = O.round_to(O.cfg_fill((batch - 1) * sa + M * N, 2, 0, O.NORMAL, 0.0, 0.02), L.F16)
    x_h = O.round_to(O.cfg_fill(batch * N, 2, 1, O.NORMAL, 0.0, 1.0), L.F16)
    raw = torch.empty(A_h.nbytes + PAGE, dtype=torch.uint8, device="cuda")
    off = (-raw.data_ptr()) % PAGE
    A = raw[off: off + A_h.nbytes]
    A.copy_(to_dev(A_h).view(torch.uint8).reshape(-1))
    x = to_dev(x_h)
    plan = L.GemvPlan(A, M, N, L.F16, L.F16, batch=batch, stride_a=sa)
    assert plan.stats()["tma"] == 0
    y64 = np.concatenate([O.gemv_f64(A_h[b * sa: b * sa + M * N], x_h[b * N:(b + 1) * N], L.F16, M, N)
                          for b in range(batch)])
    for m in ALL_MODES:
        y = torch.full((batch * M,), -1, dtype=torch.int16, device="cuda")
        plan.gemv(A, x, y, m)
        torch.cuda.synchronize()
        got = O.widen(y.cpu().numpy().view(np.uint16), L.F16)
        assert O.rel_l2(O.round_out(y64, L.F16).astype(np.float64), got) <= TOL[L.F16]
    plan.close()


def test_unaligned_rows_fall_back_to_register_kernels(dev):
    M, N = 500, 1000  # 2000-byte fp16 rows: not on 4 KiB granules
    A, x = inputs(M, N, L.F16)
    outs, stats = run(A, x, M, N, L.F16, L.F16, ALL_MODES)
    assert stats["tma"] == 0
    ref = oracle(A, x, L.F16, M, N, 1, L.F16)
    for m in ALL_MODES:
        assert O.rel_l2(ref.astype(np.float64), outs[m]) <= TOL[L.F16]


def test_back_to_back_calls_of_two_plans(dev):
    """Calls of two plans alternate back to back on one stream, x of the second written by a copy
    between them: every result matches its own plan's result from a lone call."""
    shapes = [(2048, 8192, L.F16), (1024, 4096, L.BF16)]
    plans, mats, xs, lone = [], [], [], []
    for i, (M, N, dt) in enumerate(shapes):
        A_h, x_h = inputs(M, N, dt)
        raw = torch.empty(A_h.nbytes + PAGE, dtype=torch.uint8, device="cuda")
        off = (-raw.data_ptr()) % PAGE
        A = raw[off: off + A_h.nbytes]
        A.copy_(to_dev(A_h).view(torch.uint8).reshape(-1))
        x = to_dev(x_h)
        plan = L.GemvPlan(A, M, N, dt, L.F32)
        y = torch.empty(M, dtype=torch.float32, device="cuda")
        plan.gemv(A, x, y, L.MODE_AWARE)
        torch.cuda.synchronize()
        plans.append(plan); mats.append((raw, A)); xs.append(x); lone.append(y)
    x2 = torch.empty_like(xs[1])
    outs = [[torch.empty_like(lone[i]) for _ in range(4)] for i in range(2)]
    torch.cuda.synchronize()
    for k in range(4):
        plans[0].gemv(mats[0][1], xs[0], outs[0][k], L.MODE_AWARE)
        x2.copy_(xs[1])
        plans[1].gemv(mats[1][1], x2, outs[1][k], L.MODE_AWARE)
    torch.cuda.synchronize()
    for i in range(2):
        for k in range(4):
            assert torch.equal(outs[i][k], lone[i]), f"plan {i} call {k}"
        assert plans[i].stats()["device_errors"] == 0
        plans[i].close()
