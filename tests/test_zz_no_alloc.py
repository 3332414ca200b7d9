"""The allocation-free GEMV entry point, l2d_gemv_noalloc, against the planned entry point.

Callers that cannot allocate device memory at call time -- a serving runtime that reserved all
HBM for its own pools at start-up, code running inside a CUDA stream capture, a latency-critical
path that must not enter the allocator -- call l2d_gemv_noalloc, whose scratch is a static device
array inside the library.  This test calls it through the C ABI twice in a row for every mode and
checks each result against l2d_gemv on the same inputs, within the fp16 tolerance the other GPU
tests use (relative L2 <= 2e-3).  The file is named so that pytest collects it last.
"""
import ctypes as C

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import l2domain_b200 as L  # noqa: E402

PAGE = 2 * 1024 * 1024
TOL = 2e-3


def rel_l2(ref, got):
    ref = ref.astype(np.float64)
    got = got.astype(np.float64)
    return float(np.linalg.norm(got - ref) / np.linalg.norm(ref))


def as_f32(y):
    return y.view(torch.float16).float().cpu().numpy()


def test_noalloc_matches_planned_gemv_twice_per_mode():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    torch.cuda.set_device(0)
    M, N = 3000, 8192
    nbytes = M * N * 2
    region = (nbytes + PAGE - 1) // PAGE * PAGE
    raw = torch.empty(region + PAGE, dtype=torch.uint8, device="cuda")
    off = (-raw.data_ptr()) % PAGE
    A = raw[off: off + region]
    L.fill_cfg(A, L.F16, M * N, 3, 0, 1, 0.0, 0.02)
    x = torch.empty(N * 2, dtype=torch.uint8, device="cuda")
    L.fill_cfg(x, L.F16, N, 3, 1, 1, 0.0, 1.0)
    torch.cuda.synchronize()

    plan = L.GemvPlan(A, M, N, L.F16, L.F16)
    sm = L.get_map_smid2side(0)
    mask, attr = L.get_map_memory_attr(A.data_ptr(), region, sm, 0)
    sm_arr = (C.c_int * len(sm))(*sm)
    attr_arr = (C.c_int * len(attr))(*attr)
    dmap = L.DomainMap(num_sm=len(sm), sm_domain=sm_arr, mask=mask, attr=attr_arr, num_pages=len(attr),
                       base=A.data_ptr())
    desc = L.GemvDesc(M=M, N=N, lda=0, dtype_in=L.F16, dtype_out=L.F16, batch=1, stride_a=0, stride_x=0,
                      stride_y=0, device=0, A=A.data_ptr(), flags=0)
    lib = L.lib()
    for mode in (L.MODE_AWARE, L.MODE_SWAPPED, L.MODE_OBLIVIOUS, L.MODE_STREAM):
        y_ref = torch.full((M,), -1, dtype=torch.int16, device="cuda")
        plan.gemv(A, x, y_ref, mode)
        torch.cuda.synchronize()
        ref = as_f32(y_ref)
        for call in range(2):
            y = torch.full((M,), -1, dtype=torch.int16, device="cuda")
            st = lib.l2d_gemv_noalloc(C.byref(desc), C.byref(dmap), x.data_ptr(), y.data_ptr(), mode, None)
            L.check(st)
            torch.cuda.synchronize()
            err = rel_l2(ref, as_f32(y))
            assert err <= TOL, f"mode {mode}, call {call + 1}: rel L2 {err:.3g}"
    plan.close()


def test_noalloc_rejects_sizes_beyond_its_limit():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    lib = L.lib()
    x = torch.zeros(64, dtype=torch.float32, device="cuda")
    desc = L.GemvDesc(M=L_MAX_ROWS() + 1, N=16, lda=0, dtype_in=L.F32, dtype_out=L.F32, batch=1, stride_a=0,
                      stride_x=0, stride_y=0, device=0, A=x.data_ptr(), flags=0)
    st = lib.l2d_gemv_noalloc(C.byref(desc), None, x.data_ptr(), x.data_ptr(), L.MODE_STREAM, None)
    assert st == -1
    assert b"allocation-free limit" in lib.l2d_last_error()


def L_MAX_ROWS():
    import re
    import os

    src = open(os.path.join(L.INCLUDE_DIR, "l2d.h")).read()
    return int(re.search(r"#define L2D_NOALLOC_MAX_ROWS (\d+)", src).group(1))
