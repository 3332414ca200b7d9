"""Sided matrices (l2d_sided_*) on the GPU: the cudaMallocSided placement (utility/sidedgpu.cu:791-838)
applied to the GEMV's A.

* Layout: every granule of a row of side s is homed in L2 domain s by the probed address model, and
  holds that part of the dense row, byte for byte.
* Results: every mode against the fp64 oracle (fp32 relative L2 <= 1e-5, fp16/bf16 <= 2e-3 of the
  same rounded inputs, rounded to the output type); since each row is one warp's, granules in order,
  all modes give the same bits, equal to the dense plan's STREAM call on the same A (these shapes
  are below the size from which a dense call sums its last rows in halves).
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import l2domain_b200 as L  # noqa: E402
import oracle as O  # noqa: E402

PAGE = 2 * 1024 * 1024
TOL = {L.F32: 1e-5, L.F16: 2e-3, L.BF16: 2e-3}
MODES = [L.MODE_AWARE, L.MODE_SWAPPED, L.MODE_STREAM, L.MODE_OBLIVIOUS]
TSTORE = {L.F32: torch.float32, L.F16: torch.int16, L.BF16: torch.int16}


@pytest.fixture(scope="module", autouse=True)
def gpu():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    torch.cuda.set_device(0)


def dense(M, N, dt, seed=6):
    A_h = O.round_to(O.cfg_fill(M * N, seed, 0, O.NORMAL, 0.0, 0.02, threads=0), dt)
    x_h = O.round_to(O.cfg_fill(N, seed, 1, O.NORMAL, 0.0, 1.0), dt)
    raw = torch.empty(A_h.nbytes + PAGE, dtype=torch.uint8, device="cuda")
    off = (-raw.data_ptr()) % PAGE
    A = raw[off: off + A_h.nbytes]
    A.copy_(torch.from_numpy(A_h.view(np.int16) if dt != L.F32 else A_h).cuda().view(torch.uint8).reshape(-1))
    x = torch.from_numpy(x_h.view(np.int16) if dt != L.F32 else x_h).cuda()
    return raw, A, x, A_h, x_h


def test_sided_rows_sit_in_their_domain():
    M, N, dt = 1001, 8192, L.F16
    raw, A, x, A_h, _ = dense(M, N, dt)
    s = L.SidedMatrix(M, N, dt)
    try:
        s.pack(A)
        torch.cuda.synchronize()
        info = s.info()
        assert info["rows_side"] == [501, 500] and info["granules_per_row"] == 4
        assert info["bytes"] >= M * N * 2 and info["bytes"] % PAGE == 0
        sm = L.get_map_smid2side(0)
        mask, attr = L.get_map_memory_attr(info["base"], info["bytes"], sm, 0)
        assert mask == info["mask"]
        buf = L.device_view(info["base"], info["bytes"])
        rows = list(range(0, M, 37)) + [500, 501, M - 1]
        for r in rows:
            side = 0 if r < info["rows_side"][0] else 1
            got = []
            for j, g in enumerate(s.row_granules(r)):
                assert L.predict_addr_side(info["base"], mask, attr, g) == side, (r, j)
                off = g - info["base"]
                got.append(buf[off: off + 4096].cpu().numpy())
            want = A_h[r * N:(r + 1) * N].view(np.uint8)
            assert np.array_equal(np.concatenate(got), want), r
        # every granule of the buffer is used at most once
        used = [g for r in range(M) for g in s.row_granules(r)]
        assert len(set(used)) == len(used) == M * 4
    finally:
        s.close()


@pytest.mark.parametrize("M,N,dt,do", [
    (3000, 4096, L.F16, L.F16),    # 8 KiB rows
    (2049, 8192, L.BF16, L.BF16),  # 16 KiB rows, odd M
    (513, 16384, L.F16, L.F32),    # 32 KiB rows
    (1500, 2048, L.F32, L.F32),    # 8 KiB fp32 rows
    (20000, 1024, L.F32, L.F32),   # one granule per row
    (7, 2048, L.BF16, L.F32),      # fewer rows than warps
    (1, 8192, L.F16, L.F16),       # one row
])
def test_sided_gemv_matches_oracle_and_dense_stream(M, N, dt, do):
    raw, A, x, A_h, x_h = dense(M, N, dt)
    s = L.SidedMatrix(M, N, dt, do)
    plan = L.GemvPlan(A, M, N, dt, do, tma=True)
    try:
        s.pack(A)
        y64 = O.gemv_f64(A_h, x_h, dt, M, N)
        ref = (O.round_out(y64, do) if do != L.F32 else y64).astype(np.float64)
        y_dense = torch.full((M,), -1, dtype=TSTORE[do], device="cuda")
        plan.gemv(A, x, y_dense, L.MODE_STREAM)
        outs = {}
        for mode in MODES:
            y = torch.full((M,), -1, dtype=TSTORE[do], device="cuda")
            s.gemv(x, y, mode)
            s.gemv(x, y, mode)  # a second call on the same scratch gives the same bits
            torch.cuda.synchronize()
            outs[mode] = y
            h = y.cpu().numpy()
            got = h if do == L.F32 else O.widen(h.view(np.uint16), do)
            err = O.rel_l2(ref, got)
            assert err <= TOL[dt], f"mode {mode}: rel L2 {err:.3g}"
        for mode in MODES:
            assert torch.equal(outs[mode], y_dense), f"mode {mode} differs from the dense STREAM call"
        assert plan.stats()["device_errors"] == 0
    finally:
        s.close()
        plan.close()


def test_sided_rejects_rows_off_granules():
    with pytest.raises(L.L2DError) as e:
        L.SidedMatrix(100, 1000, L.F16)
    assert e.value.status == -7
    with pytest.raises(L.L2DError) as e:
        L.SidedMatrix(100, 2048, L.F16, device=0).gemv(None, None, 9)
    assert e.value.status == -1


@pytest.mark.parametrize("M,N,dt,do", [
    (3000, 4096, L.F16, L.F16),    # 8 KiB rows
    (513, 16384, L.F16, L.F32),    # 32 KiB rows
])
def test_pooled_sided_matrix_matches_oracle_and_dense_stream(M, N, dt, do):
    """A sided matrix on whole pages of the domain-classified pool (l2d_sided_create_pooled): the
    buffer lies inside the pool, its granules are marked used while it lives and free again after
    l2d_sided_destroy, and every mode gives the oracle's values and the dense STREAM call's bits."""
    raw, A, x, A_h, x_h = dense(M, N, dt)
    free0 = None
    s = L.SidedMatrix(M, N, dt, do, pooled=True)
    plan = L.GemvPlan(A, M, N, dt, do, tma=True)
    try:
        info = s.info()
        pool_base, pinfo = L.get_sided_pool_base(0), L.pool_info(0)
        assert pool_base <= info["base"] and info["base"] + info["bytes"] <= pool_base + pinfo["mapped_bytes"]
        free0 = sum(pinfo["free_granules"])
        s.pack(A)
        y64 = O.gemv_f64(A_h, x_h, dt, M, N)
        ref = (O.round_out(y64, do) if do != L.F32 else y64).astype(np.float64)
        y_dense = torch.full((M,), -1, dtype=TSTORE[do], device="cuda")
        plan.gemv(A, x, y_dense, L.MODE_STREAM)
        for mode in MODES:
            y = torch.full((M,), -1, dtype=TSTORE[do], device="cuda")
            s.gemv(x, y, mode)
            torch.cuda.synchronize()
            h = y.cpu().numpy()
            got = h if do == L.F32 else O.widen(h.view(np.uint16), do)
            assert O.rel_l2(ref, got) <= TOL[dt], f"mode {mode}"
            assert torch.equal(y, y_dense), f"mode {mode} differs from the dense STREAM call"
    finally:
        s.close()
        plan.close()
    assert sum(L.pool_info(0)["free_granules"]) == free0 + info["bytes"] // 4096
    L.pool_release(0)  # every granule is free again: the pool unmaps its chunks
