"""GPU parity at the full sizes of the five BASELINE configs, against the CPU oracle.

Every config runs in every mode (AWARE, OBLIVIOUS, SWAPPED, STREAM) and through both kernel
families: the plan's default pick (the granule-ring kernels wherever the shape allows them) and the
register-pipelined kernels (plans made with L2D_PLAN_NO_TMA).  The bar is north_star's: relative L2
<= 1e-5 for fp32 against the fp64 oracle, <= 2e-3 for fp16/bf16 inputs against the fp64 oracle of
the same rounded inputs rounded to the output type; config 1 also meets the reference's own rule,
max |y - y_cpu| <= 1e-3 against its sequential fp32 check loop
(applications/gemv/src/gemv_k1024_persistent_subwarp.cu:383-397, applications/gemv/run.sh:97).

* Configs 1-3 (64 MiB fp32, 32 MiB fp16, 448 MiB bf16) are checked on every row; their inputs are
  generated on the host by the oracle's generator and uploaded.
* Configs 4 and 5 (4 GiB each) are generated on the device by l2d_fill_cfg; the rows checked are
  regenerated on the host by the oracle, asserted bit-identical to the device's bytes, and the
  oracle's y of those rows is the reference.  Config 4: the first and last 256 rows of every one
  of the 32 problems plus two whole problems.  Config 5: rows at the start, the middle and the end
  (the last 2560, which hold the ring kernels' tail of half-row claims),
  once with A on a 2 MiB boundary and once 4 KiB past one, where every 64th 32 KiB row straddles two
  2 MiB pages (all of those rows are checked).
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import l2domain_b200 as L  # noqa: E402
import oracle as O  # noqa: E402

PAGE = 2 * 1024 * 1024
TOL = {L.F32: 1e-5, L.F16: 2e-3, L.BF16: 2e-3}
MODES = [L.MODE_AWARE, L.MODE_OBLIVIOUS, L.MODE_SWAPPED, L.MODE_STREAM]
KERNELS = [("default", None), ("register", False)]
TSTORE = {L.F32: torch.float32, L.F16: torch.int16, L.BF16: torch.int16}


@pytest.fixture(scope="module", autouse=True)
def gpu():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    torch.cuda.set_device(0)
    yield
    torch.cuda.empty_cache()


def aligned(nbytes, offset=0):
    raw = torch.empty(nbytes + PAGE + offset, dtype=torch.uint8, device="cuda")
    o = (-raw.data_ptr()) % PAGE + offset
    return raw, raw[o: o + nbytes]


def to_dev_bytes(a):
    if a.dtype == np.uint16:
        a = a.view(np.int16)
    return torch.from_numpy(np.ascontiguousarray(a)).cuda().view(torch.uint8).reshape(-1)


def host_values(n, stream, dist, dt, first=0):
    return O.round_to(O.cfg_fill(n, 0, stream, *dist, first=first, threads=0), dt)


def widen_y(y_dev, dt):
    h = y_dev.cpu().numpy()
    return h.astype(np.float64) if dt == L.F32 else O.widen(h.view(np.uint16), dt).astype(np.float64)


def ref_out(y64, dt):
    return (y64 if dt == L.F32 else O.round_out(y64, dt)).astype(np.float64)


def run_modes(A, x, M, N, dt, batch, tma, calls=1):
    """{mode: y (float64, all rows)} from one plan; `calls` back-to-back calls per mode (the last is
    returned and must equal the first bit for bit)."""
    plan = L.GemvPlan(A, M, N, dt, dt, batch=batch, tma=tma)
    out, kern = {}, plan.stats()["ring_modes"]
    try:
        for mode in MODES:
            y = torch.full((batch * M,), -1, dtype=TSTORE[dt], device="cuda")
            plan.gemv(A, x, y, mode)
            if calls > 1:
                first = y.clone()
                for _ in range(calls - 1):
                    plan.gemv(A, x, y, mode)
                torch.cuda.synchronize()
                assert torch.equal(first, y), f"mode {mode}: repeated calls differ"
            torch.cuda.synchronize()
            out[mode] = widen_y(y, dt)
        st = plan.stats()
        assert st["device_errors"] == 0
    finally:
        plan.close()
    return out, kern


def check_rows(out, ref, rows, dt, what):
    for mode, y in out.items():
        err = O.rel_l2(ref, y[rows].astype(np.float32))
        assert err <= TOL[dt], f"{what} mode {mode}: rel L2 {err:.3g} > {TOL[dt]}"


# ---------------------------------------------------------------------------------------------
# Configs 1-3: every row
# ---------------------------------------------------------------------------------------------

FULL = {
    # name: (M, N, dtype, A dist, x dist, back-to-back calls)
    "cfg1_fp32_4096x4096": (4096, 4096, L.F32, (O.UNIFORM, -1.0, 1.0), (O.UNIFORM, -1.0, 1.0), 1),
    "cfg2_fp16_4096x4096_repeated": (4096, 4096, L.F16, (O.NORMAL, 0.0, 0.02), (O.NORMAL, 0.0, 1.0), 50),
    "cfg3_bf16_28672x8192": (28672, 8192, L.BF16, (O.NORMAL, 0.0, 0.02), (O.NORMAL, 0.0, 1.0), 1),
}


@pytest.mark.parametrize("kernels", [k for k, _ in KERNELS])
@pytest.mark.parametrize("cfg", sorted(FULL))
def test_full_config_every_row(cfg, kernels):
    M, N, dt, adist, xdist, calls = FULL[cfg]
    tma = dict(KERNELS)[kernels]
    A_h = host_values(M * N, 0, adist, dt)
    x_h = host_values(N, 1, xdist, dt)
    raw, A = aligned(A_h.nbytes)
    A.copy_(to_dev_bytes(A_h))
    x = to_dev_bytes(x_h)
    out, ring_modes = run_modes(A, x, M, N, dt, 1, tma, calls)
    if kernels == "default":
        assert ring_modes == 0b1111, "the default plan runs the granule-ring kernels at this shape"
    else:
        assert ring_modes == 0
    y64 = O.gemv_f64(A_h, x_h, dt, M, N)
    check_rows(out, ref_out(y64, dt), np.arange(M), dt, cfg)
    if dt == L.F32:  # the reference's rule against its own sequential fp32 check loop
        yseq = O.gemv_seq(A_h, x_h, dt, M, N).astype(np.float64)
        for mode, y in out.items():
            assert float(np.max(np.abs(y - yseq))) <= 1e-3, f"mode {mode}"
    del raw, A


# ---------------------------------------------------------------------------------------------
# Configs 4 and 5: 4 GiB on the device, oracle on sampled rows
# ---------------------------------------------------------------------------------------------

def sampled_oracle(A_dev, x_h, rows, N, dt, adist, M, row_first_elem):
    """Regenerates the given global rows on the host (oracle generator), asserts they equal the
    device bytes, and returns the oracle's y64 of those rows (rows of problem b use x[b])."""
    eb = L.ELEM_BYTES[dt]
    ys = []
    # contiguous runs of rows: one host generation and one device read per run
    runs = np.split(rows, np.where(np.diff(rows) != 1)[0] + 1)
    for run in runs:
        r0, nr = int(run[0]), len(run)
        host = host_values(nr * N, 0, adist, dt, first=row_first_elem(r0))
        dev = A_dev[r0 * N * eb:(r0 + nr) * N * eb].cpu().numpy().view(host.dtype)
        assert np.array_equal(dev, host), f"device rows {r0}..{r0 + nr - 1} differ from the oracle generator"
        for b in np.unique(run // M):
            sel = (run // M) == b
            sub = host.reshape(nr, N)[sel].reshape(-1)
            ys.append(O.gemv_f64(sub, x_h[b * N:(b + 1) * N], dt, int(sel.sum()), N))
    return np.concatenate(ys)


@pytest.mark.parametrize("kernels", [k for k, _ in KERNELS])
def test_cfg4_batched_32x8192x8192(kernels):
    B, M, N, dt = 32, 8192, 8192, L.F16
    adist, xdist = (O.UNIFORM, -0.05, 0.05), (O.NORMAL, 0.0, 1.0)
    tma = dict(KERNELS)[kernels]
    raw, A = aligned(B * M * N * 2)
    L.fill_cfg(A, dt, B * M * N, 0, 0, *adist)
    x_h = host_values(B * N, 1, xdist, dt)
    x = to_dev_bytes(x_h)
    torch.cuda.synchronize()
    out, _ = run_modes(A, x, M, N, dt, B, tma)
    rows = np.concatenate([np.r_[b * M: b * M + 256, (b + 1) * M - 256: (b + 1) * M] for b in range(B)] +
                          [np.arange(5 * M, 6 * M), np.arange(26 * M, 27 * M)])
    rows = np.unique(rows)
    ref = ref_out(sampled_oracle(A, x_h, rows, N, dt, adist, M, lambda r: r * N), dt)
    check_rows(out, ref, rows, dt, "cfg4")
    del raw, A


@pytest.mark.parametrize("offset", [0, 4096])
@pytest.mark.parametrize("kernels", [k for k, _ in KERNELS])
def test_cfg5_4gib_sampled_rows(kernels, offset):
    M, N, dt = 131072, 16384, L.F16
    adist, xdist = (O.NORMAL, 0.0, 0.02), (O.NORMAL, 0.0, 1.0)
    tma = dict(KERNELS)[kernels]
    raw, A = aligned(M * N * 2, offset)
    L.fill_cfg(A, dt, M * N, 0, 0, *adist)
    x_h = host_values(N, 1, xdist, dt)
    x = to_dev_bytes(x_h)
    torch.cuda.synchronize()
    out, ring_modes = run_modes(A, x, M, N, dt, 1, tma)
    if kernels == "default":
        assert ring_modes == 0b1111
    # the end: the last 2560 rows cover the ring kernels' tail (rows claimed half a row at a time)
    rows = [np.arange(0, 256), np.arange(M // 2 - 128, M // 2 + 128), np.arange(M - 2560, M)]
    if offset:
        row_bytes = N * 2
        start = offset + np.arange(M, dtype=np.int64) * row_bytes
        crossing = np.where(start // PAGE != (start + row_bytes - 1) // PAGE)[0]
        assert len(crossing) == M // 64
        rows.append(crossing)
    rows = np.unique(np.concatenate(rows))
    ref = ref_out(sampled_oracle(A, x_h, rows, N, dt, adist, M, lambda r: r * N), dt)
    check_rows(out, ref, rows, dt, f"cfg5 offset {offset}")
    del raw, A
