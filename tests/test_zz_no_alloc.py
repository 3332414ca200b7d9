"""The allocation-free GEMV entry point, l2d_gemv_noalloc, through the C ABI.

Some callers cannot call cudaMalloc when they run a GEMV: a serving runtime that reserved all HBM
for its own pools at start-up and forbids later allocations, or a latency-critical path that must
not enter the allocator.  They call l2d_gemv_noalloc, whose scratch is a static device array
inside the library.  For every dtype, for one problem and for a strided batch of three, and in
every mode, this test calls it twice in a row and checks each result against the planned entry
point l2d_gemv on the same inputs and against the CPU oracle (fp64 accumulation of the same
rounded inputs), within the tolerances the other GPU tests use: relative L2 <= 1e-5 for fp32 and
<= 2e-3 for fp16/bf16.  The file is named so that pytest collects it last.
"""
import ctypes as C
import os
import re

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import l2domain_b200 as L  # noqa: E402
import oracle as O  # noqa: E402

PAGE = 2 * 1024 * 1024
TOL = {L.F32: 1e-5, L.F16: 2e-3, L.BF16: 2e-3}
MODES = (L.MODE_AWARE, L.MODE_SWAPPED, L.MODE_OBLIVIOUS, L.MODE_STREAM)


def _gpu():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    torch.cuda.set_device(0)


def _to_dev(a):
    if a.dtype == np.uint16:
        a = a.view(np.int16)
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _host_y(y, dt_out):
    h = y.cpu().numpy()
    return h if dt_out == L.F32 else O.widen(h.view(np.uint16), dt_out)


# (dtype, M, N, batch, lda, stride_a, stride_x, stride_y); 0 = the default stride
CASES = [
    (L.F16, 3000, 8192, 1, 0, 0, 0, 0),
    (L.BF16, 1500, 8192, 1, 0, 0, 0, 0),
    (L.F32, 1200, 4096, 1, 0, 0, 0, 0),
    (L.F16, 700, 4096, 3, 4096 + 64, 700 * (4096 + 64) + 2048, 4096 + 32, 700 + 16),
    (L.BF16, 500, 2048, 3, 2048 + 8, 500 * (2048 + 8) + 520, 2048 + 8, 500 + 3),
    (L.F32, 600, 1024, 3, 1024 + 4, 600 * (1024 + 4) + 4, 1024 + 4, 600 + 5),
]


@pytest.mark.parametrize("dt,M,N,batch,lda,sa,sx,sy", CASES)
def test_noalloc_matches_planned_gemv_and_oracle_twice(dt, M, N, batch, lda, sa, sx, sy):
    _gpu()
    lda_e, sa_e = lda or N, sa or M * (lda or N)
    sx_e, sy_e = sx or N, sy or M
    eb = L.ELEM_BYTES[dt]
    n_a = (batch - 1) * sa_e + M * lda_e
    n_x = (batch - 1) * sx_e + N
    A_h = O.round_to(O.cfg_fill(n_a, 3, 0, O.NORMAL, 0.0, 0.02), dt)
    x_h = O.round_to(O.cfg_fill(n_x, 3, 1, O.NORMAL, 0.0, 1.0), dt)
    y64 = np.concatenate([O.gemv_f64(A_h[b * sa_e: b * sa_e + M * lda_e], x_h[b * sx_e: b * sx_e + N], dt, M, N,
                                     lda_e) for b in range(batch)])
    want = O.round_out(y64, dt) if dt != L.F32 else y64

    nbytes = n_a * eb
    region = (nbytes + PAGE - 1) // PAGE * PAGE
    raw = torch.empty(region + PAGE, dtype=torch.uint8, device="cuda")
    off = (-raw.data_ptr()) % PAGE
    A = raw[off: off + region]
    A[:nbytes].copy_(_to_dev(A_h).view(torch.uint8).reshape(-1))
    x = _to_dev(x_h)
    torch.cuda.synchronize()

    plan = L.GemvPlan(A, M, N, dt, dt, lda=lda, batch=batch, stride_a=sa, stride_x=sx, stride_y=sy)
    sm = L.get_map_smid2side(0)
    mask, attr = L.get_map_memory_attr(A.data_ptr(), region, sm, 0)
    sm_arr = (C.c_int * len(sm))(*sm)
    attr_arr = (C.c_int * len(attr))(*attr)
    dmap = L.DomainMap(num_sm=len(sm), sm_domain=sm_arr, mask=mask, attr=attr_arr, num_pages=len(attr),
                       base=A.data_ptr())
    desc = L.GemvDesc(M=M, N=N, lda=lda, dtype_in=dt, dtype_out=dt, batch=batch, stride_a=sa, stride_x=sx,
                      stride_y=sy, device=0, A=A.data_ptr(), flags=0)
    lib = L.lib()
    n_y = (batch - 1) * sy_e + M
    tdt = torch.float32 if dt == L.F32 else torch.int16
    rows = np.concatenate([np.arange(b * sy_e, b * sy_e + M) for b in range(batch)])
    try:
        for mode in MODES:
            y_plan = torch.full((n_y,), -1, dtype=tdt, device="cuda")
            plan.gemv(A, x, y_plan, mode)
            torch.cuda.synchronize()
            ref = _host_y(y_plan, dt)[rows]
            for call in range(2):
                y = torch.full((n_y,), -1, dtype=tdt, device="cuda")
                st = lib.l2d_gemv_noalloc(C.byref(desc), C.byref(dmap), x.data_ptr(), y.data_ptr(), mode, None)
                L.check(st)
                torch.cuda.synchronize()
                got = _host_y(y, dt)[rows]
                e_plan = O.rel_l2(ref.astype(np.float64), got)
                e_orc = O.rel_l2(want.astype(np.float64), got)
                assert e_plan <= TOL[dt], f"mode {mode}, call {call + 1}: rel L2 vs l2d_gemv {e_plan:.3g}"
                assert e_orc <= TOL[dt], f"mode {mode}, call {call + 1}: rel L2 vs oracle {e_orc:.3g}"
    finally:
        plan.close()


def _max_rows():
    src = open(os.path.join(L.INCLUDE_DIR, "l2d.h")).read()
    return int(re.search(r"#define L2D_NOALLOC_MAX_ROWS (\d+)", src).group(1))


def test_noalloc_rejects_sizes_beyond_its_limit():
    _gpu()
    lib = L.lib()
    x = torch.zeros(64, dtype=torch.float32, device="cuda")
    desc = L.GemvDesc(M=_max_rows() + 1, N=16, lda=0, dtype_in=L.F32, dtype_out=L.F32, batch=1, stride_a=0,
                      stride_x=0, stride_y=0, device=0, A=x.data_ptr(), flags=0)
    st = lib.l2d_gemv_noalloc(C.byref(desc), None, x.data_ptr(), x.data_ptr(), L.MODE_STREAM, None)
    assert st == -1
    assert b"allocation-free limit" in lib.l2d_last_error()
