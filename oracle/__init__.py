"""CPU oracle for the L2-domain-aware GEMV -- TEST INFRASTRUCTURE ONLY.

ctypes binding of ``oracle/liboracle.so`` (built by ``make -C oracle``).  Only ``tests/``,
``__graft_entry__.smoke()`` and the ``cpu_baseline`` leg of ``bench.py`` import this module; the
product library never does.  Each function cites the reference code it restates.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")
REF_PIN_PATH = os.path.join(HERE, "_ref", "libref_pin.so")

F32, F16, BF16 = 0, 1, 2
UNIFORM, NORMAL = 0, 1
DTYPE_CODE = {"fp32": F32, "fp16": F16, "bf16": BF16}
STORAGE = {F32: np.float32, F16: np.uint16, BF16: np.uint16}

_lib = None


def build() -> None:
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = C.CDLL(LIB_PATH)
        vp, i64, u64, u32 = C.c_void_p, C.c_int64, C.c_uint64, C.c_uint32
        L.or_mix32.restype = u32
        L.or_mix32.argtypes = [u32]
        L.or_ref_fill.argtypes = [vp, u64, u64, u32, C.c_int, C.c_int]
        L.or_splitmix64.restype = u64
        L.or_splitmix64.argtypes = [u64]
        L.or_rng_u64.restype = u64
        L.or_rng_u64.argtypes = [u64, u64, u64, u32]
        L.or_log_pos.restype = C.c_double
        L.or_log_pos.argtypes = [C.c_double]
        L.or_cos_2pi.restype = C.c_double
        L.or_cos_2pi.argtypes = [C.c_double]
        L.or_cfg_value.restype = C.c_float
        L.or_cfg_value.argtypes = [u64, u64, u64, C.c_int, C.c_float, C.c_float]
        L.or_cfg_fill.argtypes = [vp, u64, u64, u64, u64, C.c_int, C.c_float, C.c_float]
        L.or_cfg_fill_mt.argtypes = [vp, u64, u64, u64, u64, C.c_int, C.c_float, C.c_float, C.c_int]
        L.or_f32_to_f16.restype = C.c_uint16
        L.or_f32_to_f16.argtypes = [C.c_float]
        L.or_f16_to_f32.restype = C.c_float
        L.or_f16_to_f32.argtypes = [C.c_uint16]
        L.or_f32_to_bf16.restype = C.c_uint16
        L.or_f32_to_bf16.argtypes = [C.c_float]
        L.or_bf16_to_f32.restype = C.c_float
        L.or_bf16_to_f32.argtypes = [C.c_uint16]
        L.or_round_array.argtypes = [vp, vp, u64, C.c_int]
        L.or_widen_array.argtypes = [vp, vp, u64, C.c_int]
        L.or_gemv_seq_f32.argtypes = [vp, vp, vp, i64, i64, i64]
        L.or_gemv_seq_any.argtypes = [vp, C.c_int, vp, vp, i64, i64, i64]
        L.or_gemv_omp_any.argtypes = [vp, C.c_int, vp, vp, i64, i64, i64, C.c_int]
        L.or_gemv_f64.argtypes = [vp, C.c_int, vp, vp, i64, i64, i64]
        L.or_max_threads.restype = C.c_int
        L.or_max_abs_err.restype = C.c_double
        L.or_max_abs_err.argtypes = [vp, vp, i64]
        L.or_rel_l2.restype = C.c_double
        L.or_rel_l2.argtypes = [vp, vp, i64]
        L.or_max_abs_err_f32.restype = C.c_float
        L.or_max_abs_err_f32.argtypes = [vp, vp, i64]
        L.or_predict_far.restype = C.c_int
        L.or_predict_far.argtypes = [C.c_int, u32, u64, C.c_int]
        L.or_predict_addr_side.restype = C.c_int
        L.or_predict_addr_side.argtypes = [u64, u32, vp, u64]
        L.or_partition_rows.argtypes = [u64, u64, i64, u32, vp, vp, vp, vp, vp, vp, vp, vp, vp]
        L.or_ref_smid_side.restype = C.c_int
        L.or_ref_smid_side.argtypes = [vp, C.c_int]
        L.or_ref_mask_from_exp2.restype = u32
        L.or_ref_mask_from_exp2.argtypes = [vp, vp, vp]
        _lib = L
    return _lib


def _p(a: np.ndarray) -> int:
    return a.ctypes.data


# --------------------------------------------------------------------------------------------
# generators
# --------------------------------------------------------------------------------------------

def ref_fill(n: int, seed: int, stream: int, integer_mode: bool = False, first: int = 0) -> np.ndarray:
    """gemv_k1024_persistent_subwarp.cu:118-139 (stream 0 = A, stream 1 = x)."""
    out = np.empty(n, np.float32)
    lib().or_ref_fill(_p(out), first, n, seed & 0xFFFFFFFF, stream, int(integer_mode))
    return out


def cfg_fill(n: int, seed: int, stream: int, dist: int, p0: float, p1: float, first: int = 0,
             threads: int = 1) -> np.ndarray:
    """BASELINE-config values of flat indices [first, first + n) (counter-based, so any range can be
    generated on its own); threads > 1 (or 0 = all cores) splits the range, same values."""
    out = np.empty(n, np.float32)
    if threads == 1:
        lib().or_cfg_fill(_p(out), first, n, seed, stream, dist, p0, p1)
    else:
        lib().or_cfg_fill_mt(_p(out), first, n, seed, stream, dist, p0, p1, threads)
    return out


def round_to(a32: np.ndarray, dtype: int) -> np.ndarray:
    a32 = np.ascontiguousarray(a32, np.float32)
    out = np.empty(a32.shape, STORAGE[dtype])
    lib().or_round_array(_p(a32), _p(out), a32.size, dtype)
    return out


def widen(a: np.ndarray, dtype: int) -> np.ndarray:
    a = np.ascontiguousarray(a)
    out = np.empty(a.shape, np.float32)
    lib().or_widen_array(_p(a), _p(out), a.size, dtype)
    return out


# --------------------------------------------------------------------------------------------
# GEMV oracles
# --------------------------------------------------------------------------------------------

def gemv_seq(A: np.ndarray, x: np.ndarray, dtype: int, M: int, N: int, lda: int | None = None) -> np.ndarray:
    """gemv_k1024_persistent_subwarp.cu:383-390 over dtype storage widened to fp32."""
    A = np.ascontiguousarray(A)
    x = np.ascontiguousarray(x)
    y = np.empty(M, np.float32)
    lib().or_gemv_seq_any(_p(A), dtype, _p(x), _p(y), M, N, lda or N)
    return y


def gemv_threads(A: np.ndarray, x: np.ndarray, dtype: int, M: int, N: int, lda: int | None = None,
                 threads: int = 0) -> np.ndarray:
    A = np.ascontiguousarray(A)
    x = np.ascontiguousarray(x)
    y = np.empty(M, np.float32)
    lib().or_gemv_omp_any(_p(A), dtype, _p(x), _p(y), M, N, lda or N, threads)
    return y


def gemv_f64(A: np.ndarray, x: np.ndarray, dtype: int, M: int, N: int, lda: int | None = None) -> np.ndarray:
    A = np.ascontiguousarray(A)
    x = np.ascontiguousarray(x)
    y = np.empty(M, np.float64)
    lib().or_gemv_f64(_p(A), dtype, _p(x), _p(y), M, N, lda or N)
    return y


def max_threads() -> int:
    return int(lib().or_max_threads())


def rel_l2(ref64: np.ndarray, y: np.ndarray) -> float:
    ref64 = np.ascontiguousarray(ref64, np.float64)
    y = np.ascontiguousarray(y, np.float32)
    return float(lib().or_rel_l2(_p(ref64), _p(y), y.size))


def max_abs(ref64: np.ndarray, y: np.ndarray) -> float:
    ref64 = np.ascontiguousarray(ref64, np.float64)
    y = np.ascontiguousarray(y, np.float32)
    return float(lib().or_max_abs_err(_p(ref64), _p(y), y.size))


def round_out(y64: np.ndarray, dtype: int) -> np.ndarray:
    """The fp64 oracle rounded to the output storage type and widened back (fp32 values)."""
    y32 = np.ascontiguousarray(y64, np.float32) if dtype == F32 else np.asarray(y64, np.float64).astype(np.float32)
    if dtype == F32:
        return y32
    return widen(round_to(y32, dtype), dtype)


# --------------------------------------------------------------------------------------------
# predictor and placement
# --------------------------------------------------------------------------------------------

def predict_far(side: int, mask: int, addr: int, attr: int) -> int:
    """latopt.cuh:255-263."""
    return int(lib().or_predict_far(side, mask, addr, attr))


def partition_rows(base: int, row_bytes: int, M: int, mask: int, attr: np.ndarray):
    """gemv_k1024_persistent_subwarp.cu:261-273 -> (side0, side1, base0, base1) row lists."""
    attr = np.ascontiguousarray(attr, np.int32)
    bufs = [np.empty(max(M, 1), np.int32) for _ in range(4)]
    cnts = [np.zeros(1, np.int64) for _ in range(4)]
    lib().or_partition_rows(base, row_bytes, M, mask, _p(attr), _p(bufs[0]), _p(cnts[0]), _p(bufs[1]),
                            _p(cnts[1]), _p(bufs[2]), _p(cnts[2]), _p(bufs[3]), _p(cnts[3]))
    return tuple(b[: int(c[0])].copy() for b, c in zip(bufs, cnts))


def ref_smid_side(lat) -> int:
    """latopt.cuh:517-528."""
    a = np.ascontiguousarray(lat, np.uint32)
    return int(lib().or_ref_smid_side(_p(a), a.size))


def ref_mask_from_exp2(lat14):
    """latopt.cuh:732-746 -> (mask, exp2_avg, base_attr)."""
    a = np.ascontiguousarray(lat14, np.uint32)
    assert a.size == 14
    avg = np.zeros(1, np.float32)
    battr = np.zeros(1, np.int32)
    m = lib().or_ref_mask_from_exp2(_p(a), _p(avg), _p(battr))
    return int(m), float(avg[0]), int(battr[0])
