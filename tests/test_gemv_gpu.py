"""GPU parity of the libl2d GEMV (through its C ABI) against the CPU oracle.

Tolerances (north_star): fp32 relative L2 <= 1e-5 against the fp64 oracle; fp16/bf16 inputs with
fp32 accumulation relative L2 <= 2e-3 against the fp64 oracle of the same rounded inputs, rounded
to the output type.  The reference's own rule (max |y - ref| <= 1e-3, applications/gemv/run.sh:97)
is checked on its quick-preset data.  The exact-integer inputs (INTEGER_FLOAT_INPUTS) are bit-exact.
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
TORCH_STORAGE = {L.F32: torch.float32, L.F16: torch.int16, L.BF16: torch.int16}
ALL_MODES = [L.MODE_OBLIVIOUS, L.MODE_AWARE, L.MODE_SWAPPED, L.MODE_STREAM]


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    torch.cuda.set_device(0)
    return torch.device("cuda", 0)


def to_dev(a: np.ndarray):
    if a.dtype == np.uint16:
        a = a.view(np.int16)
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def aligned_empty(nbytes, align=2 * 1024 * 1024):
    """A device buffer whose start is 2 MiB aligned (as the reference's alloc_aligned, G:29-46)."""
    raw = torch.empty(nbytes + align, dtype=torch.uint8, device="cuda")
    off = (-raw.data_ptr()) % align
    return raw, raw[off: off + nbytes]


def host_inputs(M, N, dtype, lda=None, batch=1, seed=0, kind="cfg"):
    lda = lda or N
    if kind == "ref":
        A32 = O.ref_fill(batch * M * lda, 4242, 0)
        x32 = O.ref_fill(batch * N, 4242, 1)
    elif kind == "int":
        A32 = O.ref_fill(batch * M * lda, 4242, 0, integer_mode=True)
        x32 = O.ref_fill(batch * N, 4242, 1, integer_mode=True)
    else:
        A32 = O.cfg_fill(batch * M * lda, seed, 0, O.NORMAL, 0.0, 0.02)
        x32 = O.cfg_fill(batch * N, seed, 1, O.NORMAL, 0.0, 1.0)
    return O.round_to(A32, dtype), O.round_to(x32, dtype)


def oracle_y(A, x, dtype, M, N, lda, batch, dtype_out):
    ys = []
    for b in range(batch):
        Ab = A[b * M * lda:(b + 1) * M * lda]
        xb = x[b * N:(b + 1) * N]
        ys.append(O.gemv_f64(Ab, xb, dtype, M, N, lda))
    return np.concatenate(ys)


def run_gemv(A_h, x_h, M, N, dtype, dtype_out, modes, lda=None, batch=1, tma=None):
    lda = lda or N
    eb = L.ELEM_BYTES[dtype]
    raw, A = aligned_empty(max(A_h.nbytes, 16))
    A[: A_h.nbytes].copy_(to_dev(A_h).view(torch.uint8).reshape(-1)) if A_h.nbytes else None
    x = to_dev(x_h) if x_h.size else torch.zeros(8, dtype=torch.float32, device="cuda")
    plan = L.GemvPlan(A, M, N, dtype, dtype_out, lda=lda, batch=batch, tma=tma)
    outs = {}
    for mode in modes:
        if dtype_out == L.F32:
            y = torch.full((max(batch * M, 1),), float("nan"), dtype=torch.float32, device="cuda")
        else:
            y = torch.full((max(batch * M, 1),), -1, dtype=torch.int16, device="cuda")
        plan.gemv(A, x, y, mode)
        torch.cuda.synchronize()
        yh = y.cpu().numpy()[: batch * M]
        outs[mode] = yh if dtype_out == L.F32 else O.widen(yh.view(np.uint16), dtype_out)
    stats = plan.stats()
    plan.close()
    del raw
    return outs, stats


def check(outs, y64, dtype, dtype_out, modes):
    ref = O.round_out(y64, dtype_out) if dtype_out != L.F32 else y64
    for m in modes:
        err = O.rel_l2(ref.astype(np.float64), outs[m])
        assert err <= TOL[dtype], f"mode {m}: rel L2 {err:.3g} > {TOL[dtype]}"


SHAPES = [
    # (M, N, dtype_in, dtype_out, lda, batch)
    (2048, 1024, L.F32, L.F32, None, 1),    # the reference's quick case shape
    (512, 4096, L.F32, L.F32, None, 1),     # config-1 row length
    (256, 4096, L.F16, L.F16, None, 1),     # config-2 row length
    (300, 8192, L.BF16, L.BF16, None, 1),   # config-3 row length, bf16 out
    (64, 16384, L.F16, L.F32, None, 1),     # config-5 row length, fp32 out
    (4, 2048, L.F16, L.F16, None, 8),       # batched (config-4 layout), small
    (129, 1000, L.F32, L.F32, None, 1),     # ragged N, 16-byte multiple
    (77, 1003, L.F16, L.F16, 1008, 1),      # ragged N, lda > N
    (33, 3, L.F32, L.F32, 4, 1),            # tiny N
    (1, 8, L.BF16, L.F32, None, 1),         # single row
]


@pytest.mark.parametrize("M,N,dt,do,lda,batch", SHAPES)
def test_parity_all_modes(dev, M, N, dt, do, lda, batch):
    A, x = host_inputs(M, N, dt, lda=lda, batch=batch)
    outs, _ = run_gemv(A, x, M, N, dt, do, ALL_MODES, lda=lda, batch=batch)
    y64 = oracle_y(A, x, dt, M, N, lda or N, batch, do)
    check(outs, y64, dt, do, ALL_MODES)


def test_empty_shapes(dev):
    """M = 0 is a no-op; N = 0 gives y = 0 in every mode."""
    outs, _ = run_gemv(np.zeros(0, np.float32), np.zeros(0, np.float32), 0, 16, L.F32, L.F32, ALL_MODES)
    assert all(o.size == 0 for o in outs.values())
    outs, _ = run_gemv(np.zeros(0, np.float32), np.zeros(0, np.float32), 5, 0, L.F32, L.F32, ALL_MODES)
    for m in ALL_MODES:
        assert np.array_equal(outs[m], np.zeros(5, np.float32))


def test_quick_preset_reference_rule(dev):
    """Quick preset (M=2048, K=1024, seed 4242, mix32 inputs): max_abs <= 1e-3 per variant."""
    M, N = 2048, 1024
    A, x = host_inputs(M, N, L.F32, kind="ref")
    outs, _ = run_gemv(A, x, M, N, L.F32, L.F32, ALL_MODES)
    yseq = O.gemv_seq(A, x, O.F32, M, N)
    for m in ALL_MODES:
        assert float(np.max(np.abs(outs[m] - yseq))) <= 1e-3


def test_integer_kat_bit_exact(dev):
    g = GOLD["integer_kat"]
    M, N = g["M"], g["K"]
    A, x = host_inputs(M, N, L.F32, kind="int")
    outs, _ = run_gemv(A, x, M, N, L.F32, L.F32, ALL_MODES)
    want = np.array(g["y"], np.float32)
    for m in ALL_MODES:
        assert np.array_equal(outs[m], want), f"mode {m}"


@pytest.mark.parametrize("dt", [L.F16, L.BF16])
def test_integer_kat_half_types(dev, dt):
    """Small integers are exact in fp16/bf16 too, and so is every partial sum (|y| < 2^24)."""
    M, N = 256, 2048
    A, x = host_inputs(M, N, dt, kind="int")
    outs, _ = run_gemv(A, x, M, N, dt, L.F32, ALL_MODES)
    want = (O.widen(A, dt).reshape(M, N).astype(np.int64) @ O.widen(x, dt).astype(np.int64)).astype(np.float32)
    for m in ALL_MODES:
        assert np.array_equal(outs[m], want)


def test_aware_and_swapped_bit_identical_and_deterministic(dev):
    """Swapping which SMs take which units changes no arithmetic on split rows: the two per-row
    partials are the same sums, combined commutatively.  (AWARE also hands the bigger domain
    group an evenly spread fraction (n_big - n_small)/(n_big + n_small) of the rows whole, to
    balance unequal SM counts; SWAPPED does not, so those rows are left out.)  Repeated calls
    are bit-identical.  (The register kernels; the granule-ring kernels have their own test.)"""
    M, N = 1024, 8192
    A, x = host_inputs(M, N, L.F16)
    outs, stats = run_gemv(A, x, M, N, L.F16, L.F32, [L.MODE_AWARE, L.MODE_SWAPPED], tma=False)
    n0, n1 = stats["domain_sms"]
    num, den = abs(n1 - n0), n0 + n1
    split_rows = np.array([num == 0 or (r + 1) * num // den == r * num // den for r in range(M)])
    assert split_rows.sum() > M // 2
    assert np.array_equal(outs[L.MODE_AWARE][split_rows], outs[L.MODE_SWAPPED][split_rows])
    outs2, _ = run_gemv(A, x, M, N, L.F16, L.F32, [L.MODE_AWARE], tma=False)
    assert np.array_equal(outs[L.MODE_AWARE], outs2[L.MODE_AWARE])
    assert stats["calls"] == 2 and n0 > 0 and n1 > 0


def test_plans_of_different_sizes_coexist(dev):
    """A plan keeps working after another plan with a smaller shared-memory footprint is created
    for the same element types (the kernels' shared-memory limit is process-wide state)."""
    big_M, big_N, small_M, small_N = 512, 16384, 256, 1024
    Ab, xb = host_inputs(big_M, big_N, L.F16)
    As, xs = host_inputs(small_M, small_N, L.F16)
    raw_b, A_b = aligned_empty(Ab.nbytes)
    A_b.copy_(to_dev(Ab).view(torch.uint8).reshape(-1))
    raw_s, A_s = aligned_empty(As.nbytes)
    A_s.copy_(to_dev(As).view(torch.uint8).reshape(-1))
    x_b, x_s = to_dev(xb), to_dev(xs)
    plan_b = L.GemvPlan(A_b, big_M, big_N, L.F16, L.F32)
    plan_s = L.GemvPlan(A_s, small_M, small_N, L.F16, L.F32)
    y_b = torch.empty(big_M, device="cuda")
    y_s = torch.empty(small_M, device="cuda")
    for mode in ALL_MODES:
        plan_b.gemv(A_b, x_b, y_b, mode)
        plan_s.gemv(A_s, x_s, y_s, mode)
        torch.cuda.synchronize()
        check({mode: y_b.cpu().numpy()}, oracle_y(Ab, xb, L.F16, big_M, big_N, big_N, 1, L.F32), L.F16, L.F32, [mode])
        check({mode: y_s.cpu().numpy()}, oracle_y(As, xs, L.F16, small_M, small_N, small_N, 1, L.F32), L.F16, L.F32,
              [mode])
    plan_b.close()
    plan_s.close()


def test_device_generators_match_oracle(dev):
    n = 1 << 20
    for dt in (L.F32, L.F16, L.BF16):
        t = torch.empty(n * 2, dtype=torch.uint8, device="cuda") if dt != L.F32 else torch.empty(n, device="cuda")
        L.fill_ref(t, dt, n, 4242, 0, first=3 << 20)
        torch.cuda.synchronize()
        got = t.cpu().numpy().view(np.float32 if dt == L.F32 else np.uint16)
        assert np.array_equal(got, O.round_to(O.ref_fill(n, 4242, 0, first=3 << 20), dt))
        for dist, p0, p1 in ((O.UNIFORM, -1.0, 1.0), (O.NORMAL, 0.0, 0.02)):
            L.fill_cfg(t, dt, n, 7, 3, dist, p0, p1, first=12345)
            torch.cuda.synchronize()
            got = t.cpu().numpy().view(np.float32 if dt == L.F32 else np.uint16)
            want = O.round_to(O.cfg_fill(n, 7, 3, dist, p0, p1, first=12345), dt)
            assert np.array_equal(got, want), (dt, dist, int(np.sum(got != want)))


def test_errors_are_reported_not_fatal(dev):
    raw, A = aligned_empty(64 * 1024 * 4)
    plan = L.GemvPlan(A, 64, 1024, L.F32)
    x = torch.zeros(1024 + 4, device="cuda")
    y = torch.zeros(64, device="cuda")
    with pytest.raises(L.L2DError) as e:
        plan.gemv(A[16:], x, y)  # not the planned allocation
    assert e.value.status == -1
    with pytest.raises(L.L2DError) as e:
        plan.gemv(A, x[1:], y)  # x misaligned
    assert e.value.status == -7
    with pytest.raises(L.L2DError):
        plan.gemv(A, x, y, mode=9)
    plan.gemv(A, x, y, L.MODE_AWARE)  # still usable
    torch.cuda.synchronize()
    plan.close()
    stream_only = L.GemvPlan(A, 64, 1024, L.F32, probe=False)
    with pytest.raises(L.L2DError) as e:
        stream_only.gemv(A, x, y, L.MODE_AWARE)
    assert e.value.status == -7
    stream_only.gemv(A, x, y, L.MODE_STREAM)
    torch.cuda.synchronize()


def test_l2_flush_and_device_info(dev):
    info = L.device_info(0)
    assert info["num_sm"] > 0 and info["l2_bytes"] > 0
    L.l2_flush(0)
    torch.cuda.synchronize()
