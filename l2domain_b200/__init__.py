"""l2domain_b200 -- B200-native, L2-domain-aware GEMV (y = A.x).

Python mirror of the reference's probe/GEMV interface over the C ABI of ``lib/libl2d.so``
(declared in ``include/l2d.h``).  Names follow the reference where one exists:

* :func:`get_map_smid2side`          -- utility/latopt.cuh:532  (``get_map_smid2side<T>``)
* :func:`get_map_memory_attr`        -- utility/latopt.cuh:784  (``get_map_memory_attr<T>``)
* :func:`predict_map_memory_attr_far` -- utility/latopt.cuh:255-263
* :func:`predict_addr_side`          -- applications/gemv/src/gemv_k1024_persistent_subwarp.cu:105-108
* :func:`partition_rows`             -- same file :261-273
* :class:`GemvPlan`                  -- build_side_info + the kernel launches (:73-103, :163-231, :301-334)

Errors raise :class:`L2DError` (the reference aborts the process instead).  There is no CPU
fallback: importing this package without the built library raises immediately.
"""
from __future__ import annotations

import ctypes as C
import os
from dataclasses import dataclass
from typing import Optional, Sequence

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "lib", "libl2d.so")
INCLUDE_DIR = os.path.join(os.path.dirname(HERE), "include")

F32, F16, BF16 = 0, 1, 2
DTYPES = {"fp32": F32, "fp16": F16, "bf16": BF16}
ELEM_BYTES = {F32: 4, F16: 2, BF16: 2}
MODE_OBLIVIOUS, MODE_AWARE, MODE_SWAPPED, MODE_STREAM = 0, 1, 2, 3
MODES = {"oblivious": MODE_OBLIVIOUS, "baseline": MODE_OBLIVIOUS, "aware": MODE_AWARE,
         "swapped": MODE_SWAPPED, "stream": MODE_STREAM}
PLAN_NO_PROBE = 1
PLAN_TMA = 2      # granule-ring kernels for every mode (when the shape allows them)
PLAN_NO_TMA = 4   # register kernels only; default: picked per call
PLAN_GRANULES = 8  # split modes place 4 KiB granules by domain (rows that span both are summed in two parts)
PLAN_ROWS = 16     # split modes place whole rows by their first granule's domain (the reference's rule)
PAGE_BYTES = 2 * 1024 * 1024

OK = 0
STATUS_NAMES = {0: "L2D_OK", -1: "L2D_ERR_INVALID", -2: "L2D_ERR_CUDA", -3: "L2D_ERR_NO_DEVICE",
                -4: "L2D_ERR_PROBE_TIMEOUT", -5: "L2D_ERR_PROBE_COVERAGE", -6: "L2D_ERR_PROBE_AMBIGUOUS",
                -7: "L2D_ERR_UNSUPPORTED", -8: "L2D_ERR_IO", -9: "L2D_ERR_NCCL", -10: "L2D_ERR_NOT_LINEAR",
                -11: "L2D_ERR_STALE"}


class L2DError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {message}")
        self.status = status


class ProbeOpts(C.Structure):
    _fields_ = [("timeout_ms", C.c_uint32), ("lines_per_sm", C.c_uint32), ("lines_per_page", C.c_uint32),
                ("mask_pages", C.c_uint32), ("reserved", C.c_uint32 * 4)]


class SmProbeReport(C.Structure):
    _fields_ = [("num_sm", C.c_int), ("leader_smid", C.c_int), ("behavior", C.c_int), ("domain_sms", C.c_int * 2),
                ("near_cycles", C.c_float), ("far_cycles", C.c_float), ("threshold", C.c_float),
                ("separation", C.c_float), ("min_agreement", C.c_float), ("device_status", C.c_uint32),
                ("elapsed_ms", C.c_double)]


class AddrProbeReport(C.Structure):
    _fields_ = [("mask", C.c_uint32), ("granule_shift", C.c_int), ("near_cycles", C.c_float),
                ("far_cycles", C.c_float), ("threshold", C.c_float), ("separation", C.c_float),
                ("mask_agreement", C.c_float), ("attr_agreement", C.c_float), ("domain1_fraction", C.c_double),
                ("device_status", C.c_uint32), ("elapsed_ms", C.c_double)]


class GemvDesc(C.Structure):
    _fields_ = [("M", C.c_int64), ("N", C.c_int64), ("lda", C.c_int64), ("dtype_in", C.c_int),
                ("dtype_out", C.c_int), ("batch", C.c_int64), ("stride_a", C.c_int64), ("stride_x", C.c_int64),
                ("stride_y", C.c_int64), ("device", C.c_int), ("A", C.c_void_p), ("flags", C.c_int)]


class DomainMap(C.Structure):
    _fields_ = [("num_sm", C.c_int), ("sm_domain", C.POINTER(C.c_int)), ("mask", C.c_uint32),
                ("attr", C.POINTER(C.c_int)), ("num_pages", C.c_size_t), ("base", C.c_void_p)]


class PlanStats(C.Structure):
    _fields_ = [("rows_total", C.c_int64), ("granule_shift", C.c_int), ("domain_bytes", C.c_int64 * 2),
                ("split_rows", C.c_int64), ("domain_sms", C.c_int * 2), ("grid", C.c_int), ("block", C.c_int),
                ("scratch_bytes", C.c_size_t), ("fallback_slots", C.c_uint64), ("calls", C.c_uint64),
                ("tma", C.c_int), ("device_errors", C.c_uint64), ("ring_modes", C.c_int),
                ("ring_whole_rows", C.c_int64), ("ring_chunk_rows", C.c_int64), ("sm_map_cached", C.c_int),
                ("placement", C.c_int), ("row_domain_bytes", C.c_int64 * 2)]


# Every symbol include/l2d.h declares, with its ctypes signature.
_vp, _i, _u32, _u64, _i64, _sz = C.c_void_p, C.c_int, C.c_uint32, C.c_uint64, C.c_int64, C.c_size_t
_pi, _pu32, _pu64, _psz = C.POINTER(C.c_int), C.POINTER(C.c_uint32), C.POINTER(C.c_uint64), C.POINTER(C.c_size_t)
SIGNATURES = {
    "l2d_version": (_i, []),
    "l2d_last_error": (C.c_char_p, []),
    "l2d_status_string": (C.c_char_p, [_i]),
    "l2d_probe_sm_domains": (_i, [_i, _pi, _i, _pi, C.POINTER(ProbeOpts)]),
    "l2d_probe_sm_domains_ex": (_i, [_i, _pi, _i, _pi, C.POINTER(ProbeOpts), C.POINTER(SmProbeReport), _pu32, _sz,
                                     _psz]),
    "l2d_probe_addr_domains": (_i, [_i, _vp, _sz, _pi, _i, _pu32, _pi, _sz, _psz, C.POINTER(ProbeOpts)]),
    "l2d_probe_addr_domains_ex": (_i, [_i, _vp, _sz, _pi, _i, _pu32, _pi, _sz, _psz, C.POINTER(ProbeOpts),
                                       C.POINTER(AddrProbeReport), _pu32, _sz, _psz]),
    "l2d_analyze_sm": (_i, [_i, _i, _pu32, _pu32, _pu32, _pi, _i, C.POINTER(SmProbeReport)]),
    "l2d_analyze_addr": (_i, [_sz, _pu64, _pu32, C.POINTER(C.c_uint8), _sz, _pu32, _pi,
                              C.POINTER(AddrProbeReport)]),
    "l2d_kmeans2": (_i, [_pu32, _sz, C.POINTER(C.c_float), C.POINTER(C.c_float), C.POINTER(C.c_float),
                         C.POINTER(C.c_float)]),
    "l2d_predict_far": (_i, [_i, _u32, _u64, _i]),
    "l2d_predict_addr_side": (_i, [_u64, _u32, _pi, _sz, _u64]),
    "l2d_partition_rows": (_i, [_u64, _u64, _i64, _u32, _pi, _sz, _vp, C.POINTER(_i64), _vp, C.POINTER(_i64), _vp,
                                C.POINTER(_i64), _vp, C.POINTER(_i64)]),
    "l2d_write_smid2side_csv": (_i, [C.c_char_p, _pi, _i]),
    "l2d_read_smid2side_csv": (_i, [C.c_char_p, _pi, _i, _pi]),
    "l2d_write_mask_csv": (_i, [C.c_char_p, _u32]),
    "l2d_read_mask_csv": (_i, [C.c_char_p, _pu32]),
    "l2d_device_key": (_i, [_i, C.c_char_p, _i]),
    "l2d_domain_cache_check": (_i, [C.c_char_p, C.c_char_p, _i, _pi, _i, _pi, _pu32]),
    "l2d_domain_cache_store": (_i, [C.c_char_p, C.c_char_p, _pi, _i, _u32]),
    "l2d_domain_cache_load": (_i, [_i, C.c_char_p, _pi, _i, _pi, _pu32]),
    "l2d_plan_create": (_i, [C.POINTER(GemvDesc), C.POINTER(DomainMap), C.POINTER(_vp)]),
    "l2d_plan_destroy": (_i, [_vp]),
    "l2d_gemv": (_i, [_vp, _vp, _vp, _vp, _i, _vp]),
    "l2d_plan_stats_get": (_i, [_vp, C.POINTER(PlanStats)]),
    "l2d_plan_domain_map": (_i, [_vp, _pi, _i, _pi, _pu32]),
    "l2d_gemv_noalloc": (_i, [C.POINTER(GemvDesc), C.POINTER(DomainMap), _vp, _vp, _i, _vp]),
    "l2d_sided_create": (_i, [C.POINTER(GemvDesc), C.POINTER(_vp)]),
    "l2d_sided_create_pooled": (_i, [C.POINTER(GemvDesc), C.POINTER(ProbeOpts), C.POINTER(_vp)]),
    "l2d_sided_pack": (_i, [_vp, _vp, _i64, _vp]),
    "l2d_gemv_sided": (_i, [_vp, _vp, _vp, _i, _vp]),
    "l2d_sided_info": (_i, [_vp, _vp]),
    "l2d_sided_row_granules": (_i, [_vp, _i64, _pu64, _i, _pi]),
    "l2d_sided_destroy": (_i, [_vp]),
    "l2d_shard_create": (_i, [_i, _i, _i, _i64, _i64, _i64, _i64, _i, _i, _u32, C.POINTER(_vp)]),
    "l2d_shard_handle": (_i, [_vp, _vp, _sz, _psz]),
    "l2d_shard_connect": (_i, [_vp, _vp, _sz]),
    "l2d_shard_buffers": (_i, [_vp, _i, C.POINTER(_vp), C.POINTER(_vp)]),
    "l2d_shard_next_parity": (_i, [_vp]),
    "l2d_gemv_sharded": (_i, [_vp, _vp, _i, _vp, _pi]),
    "l2d_shard_status": (_i, [_vp, _pu32]),
    "l2d_shard_destroy": (_i, [_vp]),
    "l2d_pool_alloc": (_i, [_i, _sz, _i, C.POINTER(ProbeOpts), _pu64, _sz, _psz]),
    "l2d_pool_free": (_i, [_i, _pu64, _sz]),
    "l2d_pool_base": (_i, [_i, C.POINTER(_vp)]),
    "l2d_pool_info": (_i, [_i, _pu64, _pu64, _pu32]),
    "l2d_pool_side": (_i, [_i, _pu64, _sz, _pi]),
    "l2d_pool_release": (_i, [_i]),
    "l2d_fill_ref": (_i, [_vp, _i, _u64, _u64, _u32, _i, _i, _vp]),
    "l2d_fill_cfg": (_i, [_vp, _i, _u64, _u64, _u64, _u64, _i, C.c_float, C.c_float, _vp]),
    "l2d_l2_flush": (_i, [_i, _vp]),
    "l2d_read_stream": (_i, [_i, _vp, _sz, _i, _vp, _sz, _vp]),
    "l2d_device_info": (_i, [_i, _pi, _pi, _pi, _pi, C.c_char_p, _i]),
}

_lib: Optional[C.CDLL] = None


def lib() -> C.CDLL:
    """Loads lib/libl2d.so (raises if it was not built: there is no fallback path)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: build it with `make -C l2domain_b200/csrc` "
                              "or __graft_entry__.build()")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def check(status: int) -> int:
    if status != OK:
        msg = lib().l2d_last_error()
        raise L2DError(status, msg.decode() if msg else "")
    return status


def _ptr(t) -> int:
    if t is None:
        return 0
    if isinstance(t, int):
        return t
    if hasattr(t, "data_ptr"):
        return int(t.data_ptr())
    raise TypeError(f"expected a device pointer (int) or a tensor, got {type(t)}")


def _stream_handle(stream) -> Optional[int]:
    if stream is None:
        return None
    if isinstance(stream, int):
        return stream
    return int(getattr(stream, "cuda_stream", 0))


# --------------------------------------------------------------------------------------------
# Probes (latopt.cuh mirrors)
# --------------------------------------------------------------------------------------------

def num_sms(device: int = 0) -> int:
    n = C.c_int(0)
    check(lib().l2d_probe_sm_domains(device, None, 0, C.byref(n), None))
    return n.value


def get_map_smid2side(device: int = 0, timeout_ms: int = 0, lines_per_sm: int = 0, with_report: bool = False,
                      with_raw: bool = False):
    """SM -> L2 domain map, ``map[smid]`` in {0, 1}, domain 0 = SM 0's (latopt.cuh:532)."""
    n = num_sms(device)
    arr = (C.c_int * n)()
    opts = ProbeOpts(timeout_ms=timeout_ms, lines_per_sm=lines_per_sm)
    rep = SmProbeReport()
    L = lines_per_sm or 48
    raw_cap = n + 3 * n * L
    raw = (C.c_uint32 * raw_cap)() if with_raw else None
    raw_len = C.c_size_t(0)
    cnt = C.c_int(0)
    st = lib().l2d_probe_sm_domains_ex(device, arr, n, C.byref(cnt), C.byref(opts), C.byref(rep), raw,
                                       raw_cap if with_raw else 0, C.byref(raw_len))
    out = [int(v) for v in arr]
    if with_raw or with_report:
        extra = {"report": report_dict(rep)}
        if with_raw:
            extra["raw"] = list(raw)[: raw_len.value]
            extra["lines"] = L
        extra["status"] = st
        extra["error"] = lib().l2d_last_error().decode() if st else ""
        return out, extra
    check(st)
    return out


def get_map_memory_attr(base, nbytes: int, smid2side: Sequence[int], device: int = 0, timeout_ms: int = 0,
                        with_report: bool = False, with_raw: bool = False):
    """(mask, attr[page]) of the 2 MiB-aligned region [base, base+nbytes) (latopt.cuh:784)."""
    sm = (C.c_int * len(smid2side))(*smid2side)
    pages = C.c_size_t(0)
    check(lib().l2d_probe_addr_domains(device, _ptr(base), nbytes, sm, len(smid2side), None, None, 0,
                                       C.byref(pages), None))
    attr = (C.c_int * max(pages.value, 1))()
    mask = C.c_uint32(0)
    opts = ProbeOpts(timeout_ms=timeout_ms)
    rep = AddrProbeReport()
    raw_cap = 3 * (pages.value * 8 + 4 * 100 + 64) if with_raw else 0
    raw = (C.c_uint32 * max(raw_cap, 1))() if with_raw else None
    raw_len = C.c_size_t(0)
    st = lib().l2d_probe_addr_domains_ex(device, _ptr(base), nbytes, sm, len(smid2side), C.byref(mask), attr,
                                         pages.value, C.byref(pages), C.byref(opts), C.byref(rep), raw, raw_cap,
                                         C.byref(raw_len))
    res = (int(mask.value), [int(v) for v in attr][: pages.value])
    if with_raw or with_report:
        extra = {"report": report_dict(rep), "status": st,
                 "error": lib().l2d_last_error().decode() if st else ""}
        if with_raw and raw_len.value <= raw_cap:
            extra["raw"] = list(raw)[: raw_len.value]
        return res, extra
    check(st)
    return res


def report_dict(rep) -> dict:
    out = {}
    for name, _ in rep._fields_:
        v = getattr(rep, name)
        out[name] = list(v) if hasattr(v, "__len__") else v
    return out


def predict_map_memory_attr_far(side: int, mask: int, addr: int, attr: int) -> int:
    """latopt.cuh:255-263: popc(lo32(addr) & mask) & 1 ^ side ^ attr."""
    return int(lib().l2d_predict_far(side, mask, addr, attr))


def predict_addr_side(base: int, mask: int, attr: Sequence[int], addr: int) -> int:
    a = (C.c_int * len(attr))(*attr)
    st = lib().l2d_predict_addr_side(base, mask, a, len(attr), addr)
    if st < 0:
        check(st)
    return st


def partition_rows(base: int, row_bytes: int, M: int, mask: int, attr: Sequence[int]):
    """(side0, side1, baseline0, baseline1) row lists (gemv_k1024_persistent_subwarp.cu:261-273)."""
    a = (C.c_int * len(attr))(*attr)
    bufs = [(C.c_int32 * max(M, 1))() for _ in range(4)]
    cnts = [C.c_int64(0) for _ in range(4)]
    check(lib().l2d_partition_rows(base, row_bytes, M, mask, a, len(attr), bufs[0], C.byref(cnts[0]), bufs[1],
                                   C.byref(cnts[1]), bufs[2], C.byref(cnts[2]), bufs[3], C.byref(cnts[3])))
    return tuple(list(b)[: c.value] for b, c in zip(bufs, cnts))


def write_smid2side_csv(path: str, sm_map: Sequence[int]) -> None:
    a = (C.c_int * len(sm_map))(*sm_map)
    check(lib().l2d_write_smid2side_csv(path.encode(), a, len(sm_map)))


def read_smid2side_csv(path: str) -> list:
    n = C.c_int(0)
    check(lib().l2d_read_smid2side_csv(path.encode(), None, 0, C.byref(n)))
    a = (C.c_int * n.value)()
    check(lib().l2d_read_smid2side_csv(path.encode(), a, n.value, C.byref(n)))
    return list(a)


def write_mask_csv(path: str, mask: int) -> None:
    check(lib().l2d_write_mask_csv(path.encode(), mask))


def read_mask_csv(path: str) -> int:
    m = C.c_uint32(0)
    check(lib().l2d_read_mask_csv(path.encode(), C.byref(m)))
    return int(m.value)


# --------------------------------------------------------------------------------------------
# Domain-map cache (utility/sidedgpu.cu:118-130, 278-300, 487-507 read the same files back)
# --------------------------------------------------------------------------------------------

def device_key(device: int = 0) -> str:
    """The identity a cached map is keyed to: GPU UUID, SM count, compute capability, driver API."""
    buf = C.create_string_buffer(512)
    check(lib().l2d_device_key(device, buf, 512))
    return buf.value.decode()


def domain_cache_store(directory: str, key: str, sm_map: Sequence[int], mask: int) -> None:
    arr = (C.c_int * len(sm_map))(*sm_map)
    check(lib().l2d_domain_cache_store(directory.encode(), key.encode(), arr, len(sm_map), mask))


def domain_cache_check(directory: str, key: Optional[str], num_sm: int = 0):
    """(sm_map, mask) from the cache in `directory` if it belongs to `key` (None: not checked) and
    has `num_sm` SMs (0: not checked); raises L2DError (L2D_ERR_IO / L2D_ERR_STALE) otherwise."""
    n = C.c_int(0)
    m = C.c_uint32(0)
    cap = 1024
    arr = (C.c_int * cap)()
    check(lib().l2d_domain_cache_check(directory.encode(), key.encode() if key is not None else None, num_sm, arr,
                                       cap, C.byref(n), C.byref(m)))
    return list(arr[: n.value]), int(m.value)


def domain_cache_load(directory: str, device: int = 0):
    """domain_cache_check against this device's key and SM count."""
    n = C.c_int(0)
    m = C.c_uint32(0)
    arr = (C.c_int * 1024)()
    check(lib().l2d_domain_cache_load(device, directory.encode(), arr, 1024, C.byref(n), C.byref(m)))
    return list(arr[: n.value]), int(m.value)


# --------------------------------------------------------------------------------------------
# GEMV plans
# --------------------------------------------------------------------------------------------

@dataclass
class DomainModel:
    sm_domain: list
    mask: int
    attr: list
    base: int


class GemvPlan:
    """A GEMV plan for one A allocation: y = A.x (batched optional), fp32 accumulation.

    ``tma``: None picks the granule-ring (TMA) or register kernels per call, True uses the rings
    for every call the shape allows, False only the register kernels.  ``placement`` ("granules",
    "rows" or None for the plan's choice): how the split modes divide A between the two domain
    groups -- granule by granule, or whole rows by the domain of their first granule."""

    def __init__(self, A, M: int, N: int, dtype_in: int = F32, dtype_out: Optional[int] = None, lda: int = 0,
                 batch: int = 1, stride_a: int = 0, stride_x: int = 0, stride_y: int = 0, device: int = 0,
                 domains: Optional[DomainModel] = None, probe: bool = True, tma: Optional[bool] = None,
                 placement: Optional[str] = None):
        self._plan = C.c_void_p(0)
        self.desc = GemvDesc(M=M, N=N, lda=lda, dtype_in=dtype_in,
                             dtype_out=dtype_in if dtype_out is None else dtype_out, batch=batch,
                             stride_a=stride_a, stride_x=stride_x, stride_y=stride_y, device=device,
                             A=_ptr(A), flags=(0 if probe else PLAN_NO_PROBE) |
                             (0 if tma is None else PLAN_TMA if tma else PLAN_NO_TMA) |
                             {None: 0, "granules": PLAN_GRANULES, "rows": PLAN_ROWS}[placement])
        dm = None
        if domains is not None:
            self._sm = (C.c_int * len(domains.sm_domain))(*domains.sm_domain)
            self._attr = (C.c_int * len(domains.attr))(*domains.attr)
            dm = DomainMap(num_sm=len(domains.sm_domain), sm_domain=self._sm, mask=domains.mask, attr=self._attr,
                           num_pages=len(domains.attr), base=domains.base)
        check(lib().l2d_plan_create(C.byref(self.desc), C.byref(dm) if dm is not None else None,
                                    C.byref(self._plan)))
        self.A_ptr = _ptr(A)

    def gemv(self, A, x, y, mode: int = MODE_AWARE, stream=None) -> None:
        check(lib().l2d_gemv(self._plan, _ptr(A), _ptr(x), _ptr(y), mode, _stream_handle(stream)))

    def stats(self) -> dict:
        s = PlanStats()
        check(lib().l2d_plan_stats_get(self._plan, C.byref(s)))
        return report_dict(s)

    def domain_map(self):
        n = C.c_int(0)
        m = C.c_uint32(0)
        check(lib().l2d_plan_domain_map(self._plan, None, 0, C.byref(n), C.byref(m)))
        a = (C.c_int * n.value)()
        check(lib().l2d_plan_domain_map(self._plan, a, n.value, C.byref(n), C.byref(m)))
        return list(a), int(m.value)

    def close(self) -> None:
        if self._plan and self._plan.value:
            check(lib().l2d_plan_destroy(self._plan))
            self._plan = C.c_void_p(0)

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class SidedInfo(C.Structure):
    _fields_ = [("rows_side", C.c_int64 * 2), ("granules_per_row", C.c_int), ("base", C.c_void_p),
                ("bytes", C.c_size_t), ("mask", C.c_uint32)]


class SidedMatrix:
    """A copy of a dense row-major M x N matrix placed by L2 domain (the cudaMallocSided placement of
    utility/sidedgpu.cu:791-838 applied to the GEMV's A): the first rows_side[0] rows live only in
    granules homed in domain 0, the rest only in domain-1 granules.  ``pack(A)`` copies A in;
    ``gemv(x, y, mode)`` computes y = A.x, in AWARE mode from near granules only.  ``pooled=True``
    takes the buffer as whole pages of the device's domain-classified pool (l2d_pool_*) instead of
    a buffer of its own."""

    def __init__(self, M: int, N: int, dtype_in: int = F16, dtype_out: Optional[int] = None, device: int = 0,
                 pooled: bool = False):
        self._s = C.c_void_p(0)
        self.M, self.N, self.device = M, N, device
        desc = GemvDesc(M=M, N=N, lda=0, dtype_in=dtype_in, dtype_out=dtype_in if dtype_out is None else dtype_out,
                        batch=1, stride_a=0, stride_x=0, stride_y=0, device=device, A=None, flags=0)
        if pooled:
            check(lib().l2d_sided_create_pooled(C.byref(desc), None, C.byref(self._s)))
        else:
            check(lib().l2d_sided_create(C.byref(desc), C.byref(self._s)))

    def pack(self, A, lda: int = 0, stream=None) -> None:
        check(lib().l2d_sided_pack(self._s, _ptr(A), lda, _stream_handle(stream)))

    def gemv(self, x, y, mode: int = MODE_AWARE, stream=None) -> None:
        check(lib().l2d_gemv_sided(self._s, _ptr(x), _ptr(y), mode, _stream_handle(stream)))

    def info(self) -> dict:
        i = SidedInfo()
        check(lib().l2d_sided_info(self._s, C.byref(i)))
        return {"rows_side": list(i.rows_side), "granules_per_row": i.granules_per_row, "base": i.base or 0,
                "bytes": i.bytes, "mask": i.mask}

    def row_granules(self, row: int) -> list:
        n = C.c_int(0)
        check(lib().l2d_sided_row_granules(self._s, row, None, 0, C.byref(n)))
        a = (C.c_uint64 * n.value)()
        check(lib().l2d_sided_row_granules(self._s, row, a, n.value, C.byref(n)))
        return list(a)

    def close(self) -> None:
        if self._s and self._s.value:
            check(lib().l2d_sided_destroy(self._s))
            self._s = C.c_void_p(0)

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class PeerShard:
    """This rank's part of a row-sharded GEMV whose x broadcast and y gather run over peer memory.

    No counterpart in the reference (it is single-GPU).  ``handle()`` gives the bytes every rank
    must receive from every other (in rank order) before ``connect(blobs)``; ``step(plan)`` runs one
    sharded GEMV: rank 0's ``x(parity)`` buffer is the input of the step, every rank's ``y(parity)``
    buffer holds all ``M_total`` rows after it.  Waits are bounded by ``timeout_ms``; ``status()``
    returns the timeout bits (1: x never arrived, 2: a peer's rows never arrived).
    """

    def __init__(self, device: int, rank: int, world: int, M_total: int, row0: int, rows: int, N: int,
                 dtype_in: int, dtype_out: int, timeout_ms: int = 2000):
        self._s = C.c_void_p(0)
        self.device, self.rank, self.world = device, rank, world
        self.M_total, self.row0, self.rows, self.N = M_total, row0, rows, N
        self._eb_in, self._eb_out = ELEM_BYTES[dtype_in], ELEM_BYTES[dtype_out]
        check(lib().l2d_shard_create(device, rank, world, M_total, row0, rows, N, dtype_in, dtype_out, timeout_ms,
                                     C.byref(self._s)))

    def handle(self) -> bytes:
        n = C.c_size_t(0)
        check(lib().l2d_shard_handle(self._s, None, 0, C.byref(n)))
        buf = C.create_string_buffer(n.value)
        check(lib().l2d_shard_handle(self._s, buf, n.value, C.byref(n)))
        return buf.raw[: n.value]

    def connect(self, blobs: Sequence[bytes]) -> None:
        if len(blobs) != self.world or len({len(b) for b in blobs}) != 1:
            raise ValueError(f"expected {self.world} blobs of one size")
        joined = b"".join(blobs)
        check(lib().l2d_shard_connect(self._s, joined, len(blobs[0])))

    def buffers(self, parity: int):
        x, y = C.c_void_p(0), C.c_void_p(0)
        check(lib().l2d_shard_buffers(self._s, parity, C.byref(x), C.byref(y)))
        return int(x.value or 0), int(y.value or 0)

    def x_tensor(self, parity: int):
        """torch uint8 view of this rank's x buffer of one parity (rank 0 writes the step's x here)."""
        return device_view(self.buffers(parity)[0], self.N * self._eb_in, self.device)

    def y_tensor(self, parity: int):
        """torch uint8 view of this rank's gathered y buffer (all M_total rows) of one parity."""
        return device_view(self.buffers(parity)[1], self.M_total * self._eb_out, self.device)

    def next_parity(self) -> int:
        return int(lib().l2d_shard_next_parity(self._s))

    def step(self, plan: "GemvPlan", mode: int = MODE_AWARE, stream=None) -> int:
        par = C.c_int(0)
        check(lib().l2d_gemv_sharded(plan._plan, self._s, mode, _stream_handle(stream), C.byref(par)))
        return par.value

    def status(self) -> int:
        v = C.c_uint32(0)
        check(lib().l2d_shard_status(self._s, C.byref(v)))
        return int(v.value)

    def close(self) -> None:
        if self._s and self._s.value:
            check(lib().l2d_shard_destroy(self._s))
            self._s = C.c_void_p(0)

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


# --------------------------------------------------------------------------------------------
# Helpers
# --------------------------------------------------------------------------------------------

# --------------------------------------------------------------------------------------------
# Domain-classified pool (utility/sidedgpu.cu:791-882 mirrors)
# --------------------------------------------------------------------------------------------

POOL_GRANULE = 4096


def malloc_sided(nbytes: int, side: int, device: int = 0, timeout_ms: int = 0) -> list:
    """cudaMallocSided: free 4 KiB granules of one L2 side, as indices from :func:`get_sided_pool_base`."""
    n = max(0, -(-nbytes // POOL_GRANULE))
    buf = (C.c_uint64 * max(n, 1))()
    got = C.c_size_t(0)
    opts = ProbeOpts(timeout_ms=timeout_ms)
    check(lib().l2d_pool_alloc(device, nbytes, side, C.byref(opts), buf, n, C.byref(got)))
    return list(buf[: got.value])


def free_sided(granules: Sequence[int], device: int = 0) -> None:
    """cudaFreeSided."""
    arr = (C.c_uint64 * max(len(granules), 1))(*granules)
    check(lib().l2d_pool_free(device, arr, len(granules)))


def get_sided_pool_base(device: int = 0) -> int:
    """cudaGetSidedPoolBase: granule g of the pool lives at base + g * 4096."""
    p = C.c_void_p(0)
    check(lib().l2d_pool_base(device, C.byref(p)))
    return int(p.value or 0)


def pool_info(device: int = 0) -> dict:
    mapped, free, mask = C.c_uint64(0), (C.c_uint64 * 2)(), C.c_uint32(0)
    check(lib().l2d_pool_info(device, C.byref(mapped), free, C.byref(mask)))
    return {"mapped_bytes": mapped.value, "free_granules": [free[0], free[1]], "mask": mask.value}


def pool_sides(granules: Sequence[int], device: int = 0) -> list:
    arr = (C.c_uint64 * max(len(granules), 1))(*granules)
    out = (C.c_int * max(len(granules), 1))()
    check(lib().l2d_pool_side(device, arr, len(granules), out))
    return list(out[: len(granules)])


def pool_release(device: int = 0) -> None:
    check(lib().l2d_pool_release(device))


class _CudaArray:
    """Minimal __cuda_array_interface__ holder, so torch can view library-owned device memory."""

    def __init__(self, ptr: int, nbytes: int):
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False),
                                         "version": 3, "strides": None}


def device_view(ptr: int, nbytes: int, device: int = 0):
    """A torch uint8 tensor sharing ``nbytes`` of device memory at ``ptr`` (no copy, not owned)."""
    import torch

    return torch.as_tensor(_CudaArray(ptr, nbytes), device=torch.device("cuda", device))


def fill_ref(dst, dtype: int, n: int, seed: int, stream_id: int, integer_mode: bool = False, first: int = 0,
             stream=None) -> None:
    check(lib().l2d_fill_ref(_ptr(dst), dtype, first, n, seed & 0xFFFFFFFF, stream_id, int(integer_mode),
                             _stream_handle(stream)))


def fill_cfg(dst, dtype: int, n: int, seed: int, rng_stream: int, dist: int, p0: float, p1: float, first: int = 0,
             stream=None) -> None:
    check(lib().l2d_fill_cfg(_ptr(dst), dtype, first, n, seed, rng_stream, dist, p0, p1, _stream_handle(stream)))


def l2_flush(device: int = 0, stream=None) -> None:
    check(lib().l2d_l2_flush(device, _stream_handle(stream)))


def read_stream(buf, nbytes: int, sink, sink_words: int, device: int = 0, stream=None, passes: int = 1) -> None:
    """Reads [buf, buf + nbytes) `passes` times in one launch (the read-bandwidth roofline helper);
    sink holds one word per SM."""
    check(lib().l2d_read_stream(device, _ptr(buf), nbytes, passes, _ptr(sink), sink_words, _stream_handle(stream)))


def device_info(device: int = 0) -> dict:
    n, l2, ma, mi = C.c_int(0), C.c_int(0), C.c_int(0), C.c_int(0)
    name = C.create_string_buffer(256)
    check(lib().l2d_device_info(device, C.byref(n), C.byref(l2), C.byref(ma), C.byref(mi), name, 256))
    return {"num_sm": n.value, "l2_bytes": l2.value, "cc": (ma.value, mi.value), "name": name.value.decode()}
