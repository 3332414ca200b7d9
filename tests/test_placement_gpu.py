"""GPU parity of the two placements of the split modes (AWARE, SWAPPED, OBLIVIOUS).

Granule placement sends every 4 KiB granule to the domain group of its domain (rows that span both
domains are summed in two parts); row placement sends every row whole to one group: the group of
the domain of its first granule (the reference's rule, gemv_k1024_persistent_subwarp.cu:264-268;
SWAPPED takes the other group, OBLIVIOUS alternates rows as the reference's baseline does, :269).
The plan picks rows for rows of up to four granules and granules above that unless the caller
forces one.  Every placement, mode and kernel family is compared with the fp64 oracle at the
north_star tolerances (fp32 relative L2 <= 1e-5, fp16/bf16 <= 2e-3); on the granule-ring kernels
a row placed whole is summed by one warp over its granules in order, so every split mode under
row placement gives STREAM's bits exactly.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import l2domain_b200 as L  # noqa: E402
import oracle as O  # noqa: E402

TOL = {L.F32: 1e-5, L.F16: 2e-3, L.BF16: 2e-3}
SPLIT_MODES = [L.MODE_OBLIVIOUS, L.MODE_AWARE, L.MODE_SWAPPED]
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


def setup(M, N, dtype, lda=None, seed=0):
    lda = lda or N
    A32 = O.cfg_fill(M * lda, seed, 0, O.NORMAL, 0.0, 0.02)
    x32 = O.cfg_fill(N, seed, 1, O.NORMAL, 0.0, 1.0)
    A_h, x_h = O.round_to(A32, dtype), O.round_to(x32, dtype)
    raw = torch.empty(A_h.nbytes + PAGE, dtype=torch.uint8, device="cuda")
    off = (-raw.data_ptr()) % PAGE
    A = raw[off: off + A_h.nbytes]
    A.copy_(to_dev(A_h).view(torch.uint8).reshape(-1))
    return raw, A, to_dev(x_h), A_h, x_h


def call(plan, A, x, M, dtype_out, mode):
    if dtype_out == L.F32:
        y = torch.full((M,), float("nan"), dtype=torch.float32, device="cuda")
    else:
        y = torch.full((M,), -1, dtype=torch.int16, device="cuda")
    plan.gemv(A, x, y, mode)
    torch.cuda.synchronize()
    yh = y.cpu().numpy()
    return yh if dtype_out == L.F32 else O.widen(yh.view(np.uint16), dtype_out)


def reference(A_h, x_h, dtype, dtype_out, M, N, lda):
    y = O.gemv_f64(A_h, x_h, dtype, M, N, lda)
    return (O.round_out(y, dtype_out) if dtype_out != L.F32 else y).astype(np.float64)


@pytest.mark.parametrize("tma", [True, False])
@pytest.mark.parametrize("placement", ["rows", "granules"])
@pytest.mark.parametrize("M,N,dtype,dtype_out", [
    (3000, 4096, L.F16, L.F16),     # 8 KiB rows
    (2049, 8192, L.BF16, L.BF16),   # 16 KiB rows
    (1500, 2048, L.F32, L.F32),     # 8 KiB fp32 rows
    (513, 16384, L.F16, L.F32),     # 32 KiB rows
])
def test_placements_match_oracle(dev, M, N, dtype, dtype_out, placement, tma):
    raw, A, x, A_h, x_h = setup(M, N, dtype)
    plan = L.GemvPlan(A, M, N, dtype, dtype_out, tma=tma, placement=placement)
    st = plan.stats()
    assert st["placement"] == (1 if placement == "rows" else 0)
    assert st["tma"] == (2 if tma else 0)
    ref = reference(A_h, x_h, dtype, dtype_out, M, N, N)
    for m in SPLIT_MODES + [L.MODE_STREAM]:
        err = O.rel_l2(ref, call(plan, A, x, M, dtype_out, m))
        assert err <= TOL[dtype], f"mode {m}: rel L2 {err:.3g}"
    assert plan.stats()["device_errors"] == 0
    plan.close()


def test_row_placement_gives_stream_bits_on_ring_kernels(dev):
    M, N = 4096, 4096
    raw, A, x, A_h, x_h = setup(M, N, L.BF16, seed=3)
    plan = L.GemvPlan(A, M, N, L.BF16, L.F32, tma=True, placement="rows")
    ys = {m: call(plan, A, x, M, L.F32, m) for m in SPLIT_MODES + [L.MODE_STREAM]}
    for m in SPLIT_MODES:
        assert np.array_equal(ys[m], ys[L.MODE_STREAM]), f"mode {m}"
    # Repeated calls give the same bits (the pools reset; nothing depends on who claimed a row).
    assert np.array_equal(call(plan, A, x, M, L.F32, L.MODE_AWARE), ys[L.MODE_AWARE])
    plan.close()


def test_row_placement_off_granule_rows_on_register_kernels(dev):
    """Rows that start inside a granule (lda not a multiple of 4 KiB) run the register kernels,
    which place each row by the domain of the 1 KiB unit holding its first element."""
    M, N, lda = 777, 3000, 3016
    raw, A, x, A_h, x_h = setup(M, N, L.F16, lda=lda, seed=5)
    plan = L.GemvPlan(A, M, N, L.F16, L.F32, lda=lda, placement="rows")
    assert plan.stats()["ring_modes"] == 0
    ref = reference(A_h, x_h, L.F16, L.F32, M, N, lda)
    for m in SPLIT_MODES:
        assert O.rel_l2(ref, call(plan, A, x, M, L.F32, m)) <= TOL[L.F16], f"mode {m}"
    plan.close()


def test_auto_placement_and_row_census(dev):
    """The plan's own choice: whole rows up to four granules a row, granules from eight; the row
    census splits the matrix's bytes between the two domains (rows alternate on B200's hash)."""
    for M, N, want in ((2048, 4096, 1), (1024, 8192, 1), (512, 16384, 0)):
        raw, A, x, A_h, x_h = setup(M, N, L.F16)
        plan = L.GemvPlan(A, M, N, L.F16, L.F16)
        st = plan.stats()
        assert st["placement"] == want, (M, N)
        rd = st["row_domain_bytes"]
        assert rd[0] + rd[1] == M * N * 2
        assert min(rd) >= 0.4 * M * N * 2
        plan.close()
