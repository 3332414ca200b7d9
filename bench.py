#!/usr/bin/env python3
"""Benchmark of the L2-domain-aware B200 GEMV (one JSON line on rank 0).

Workload (default ``cfg5``): the row-sharded fp16 GEMV of the configs -- A is M=131072 x N=16384
fp16 (4 GiB), A ~ N(0, 0.02), x ~ N(0, 1), fp32 accumulation, fp16 y.  With N GPUs each rank owns
M/N contiguous rows; one step is: x from rank 0 to every rank, the domain-aware GEMV of the rank's
shard, the y shards gathered on every rank.  The exchange runs over peer memory inside the GEMV
launch by default (``--collective p2p``: rank 0 pushes x over NVLink, and whoever stores a row's
final y also stores it into every peer's gathered y) or as NCCL broadcast + all_gather
(``--collective nccl``).  With one GPU
the step is the GEMV alone (the whole 4 GiB matrix).  Every rank's A is larger than L2 at every
N <= 8 (>= 512 MiB), so no flush is needed.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload cfg5]
                    [--collective p2p|nccl]

``--impl reference`` times the reference's CPU GEMV check loop (the oracle restatement of
applications/gemv/src/gemv_k1024_persistent_subwarp.cu:383-390) on all host cores, over a bounded
row sample of the same matrix, on rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

import numpy as np

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

METRIC = "GEMV GB/s (frac of HBM peak), µs/call; domain-aware vs naive, 1–8 B200"
FALLBACK_HBM_GBS = 6650.0
SPEC_HBM_GBS = 8000.0

F32, F16, BF16 = 0, 1, 2
UNIFORM, NORMAL = 0, 1
DT_NAME = {F32: "fp32", F16: "fp16", BF16: "bf16"}
EB = {F32: 4, F16: 2, BF16: 2}

WORKLOADS = {
    "cfg5": dict(M=131072, N=16384, batch=1, dtype=F16, a=(NORMAL, 0.0, 0.02), x=(NORMAL, 0.0, 1.0),
                 name="row-sharded fp16 GEMV, A 131072x16384 (4 GiB), x broadcast + y gather"),
    "cfg3": dict(M=28672, N=8192, batch=1, dtype=BF16, a=(NORMAL, 0.0, 0.02), x=(NORMAL, 0.0, 1.0),
                 name="bf16 LLM-decode GEMV, A 28672x8192 (448 MiB)"),
    "cfg4": dict(M=8192, N=8192, batch=32, dtype=F16, a=(UNIFORM, -0.05, 0.05), x=(NORMAL, 0.0, 1.0),
                 name="batched fp16 GEMV, 32 x (8192x8192)"),
}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="cfg5")
    ap.add_argument("--collective", choices=["p2p", "nccl"], default="p2p",
                    help="N>1: x push and y gather over peer memory inside the GEMV launch (p2p) or NCCL collectives")
    ap.add_argument("--cpu-seconds", type=float, default=10.0, help="budget of the cpu_baseline leg")
    ap.add_argument("--rows", type=int, default=0,
                    help="override M (a smaller case of the same row shape, for ncu captures)")
    ap.add_argument("--kernel", choices=["auto", "ring", "register"], default="auto",
                    help="GEMV kernels: picked per call (auto), TMA granule rings, or register pipeline")
    ap.add_argument("--no-aux", action="store_true", help="skip the per-mode and L2-resident side measurements")
    return ap.parse_args()


def dist_env():
    return (int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")),
            int(os.environ.get("LOCAL_RANK", "0")))


def measured_peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs, copy burst)"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback (6.65 TB/s earlier pool measurement)"


def profiled_traffic(workload: str, rows_local: int):
    """DRAM bytes per launch from the committed ncu summary (profiles/), scaled to this launch."""
    path = os.path.join(REPO, "profiles", f"gemv_{workload}_traffic.md")
    try:
        with open(path) as f:
            for line in f:
                if line.startswith("traffic_bytes_per_row:"):
                    return float(line.split(":")[1]) * rows_local
    except OSError:
        pass
    return None


# ------------------------------------------------------------------------------------------------
# Clock sampling (NVML) during the timed region
# ------------------------------------------------------------------------------------------------

REASON_BITS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
               0x10: "sync_boost", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
               0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting"}


class ClockSampler:
    def __init__(self, torch_dev: int, period_s: float = 0.004):
        self.samples, self.reasons, self.max_mhz, self.ok = [], 0, None, False
        self.period = period_s
        self._stop = threading.Event()
        self._t = None
        self._recording = False
        try:
            import pynvml as N
            N.nvmlInit()
            self.N = N
            self.h = None
            try:
                import torch
                p = torch.cuda.get_device_properties(torch_dev)
                bus = f"{p.pci_domain_id:08x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
                self.h = N.nvmlDeviceGetHandleByPciBusId(bus.encode())
            except Exception:
                self.h = N.nvmlDeviceGetHandleByIndex(torch_dev)
            self.max_mhz = N.nvmlDeviceGetMaxClockInfo(self.h, N.NVML_CLOCK_SM)
            self._reasons_fn = getattr(N, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                getattr(N, "nvmlDeviceGetCurrentClocksThrottleReasons")
            self.ok = True
        except Exception as e:  # noqa: BLE001 -- NVML is optional on the box
            self.err = str(e)

    def _sample(self, keep=True):
        N = self.N
        mhz = N.nvmlDeviceGetClockInfo(self.h, N.NVML_CLOCK_SM)
        reasons = int(self._reasons_fn(self.h))
        if keep:
            self.samples.append(mhz)
            self.reasons |= reasons

    def _run(self):
        while not self._stop.is_set():
            try:
                self._sample(self._recording)
            except Exception:
                pass
            time.sleep(self.period)

    def start(self):
        """Starts sampling without recording, so the thread and NVML are warm before the timed region."""
        if self.ok and self._t is None:
            self._recording = False
            self._sample(False)
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def __enter__(self):
        if self.ok:
            self.start()
            self._sample()
            self._recording = True
        return self

    def __exit__(self, *a):
        if self.ok:
            self._recording = False
            self._stop.set()
            self._t.join()
            self._sample()

    def summary(self):
        if not self.ok or not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["nvml unavailable"]}
        names = [n for b, n in REASON_BITS.items() if self.reasons & b]
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz, "reasons": names,
                "samples": len(self.samples)}


# ------------------------------------------------------------------------------------------------
# Reference arm: the reference's CPU GEMV loop on all host cores
# ------------------------------------------------------------------------------------------------

def run_reference(args, rank, world):
    if rank != 0:
        return 0
    import oracle as O
    W = WORKLOADS[args.workload]
    N, dt = W["N"], W["dtype"]
    rows = min(4096, W["M"])
    A32 = O.cfg_fill(rows * N, 0, 0, *W["a"])
    x32 = O.cfg_fill(N, 0, 1, *W["x"])
    A = O.round_to(A32, dt)
    x = O.round_to(x32, dt)
    del A32, x32
    cores = O.max_threads()
    for _ in range(args.warmup):
        O.gemv_threads(A, x, dt, rows, N, threads=cores)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        O.gemv_threads(A, x, dt, rows, N, threads=cores)
    dt_s = (time.perf_counter() - t0) / max(args.steps, 1)
    nbytes = rows * N * EB[dt] + N * EB[dt] + rows * EB[dt]
    gbs = nbytes / dt_s / 1e9
    sample = (f"rows 0..{rows - 1} of the {args.workload} matrix ({rows}x{N} {DT_NAME[dt]}, same generator and "
              f"seed), sequential fp32 dot per row (gemv_k1024_persistent_subwarp.cu:383-390), rows split over "
              f"{cores} threads")
    line = {
        "metric": METRIC, "value": round(gbs, 3), "unit": "GB/s", "impl": "reference", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt_s * 1e3, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": DT_NAME[dt], "data": "synthetic",
        "config": {"workload": args.workload, "M": W["M"], "N": N, "batch": W["batch"], "sample_rows": rows},
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": cores, "kind": "port", "sample": sample},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------------------------------------------------
# Timing helpers and the side measurements of the other configs
# ------------------------------------------------------------------------------------------------

MODE_NAMES = (("aware", 1), ("oblivious", 0), ("swapped", 2), ("stream", 3))
PLACEMENTS = ("granules", "rows")  # l2d_plan_stats.placement 0 / 1


def kernel_time_us(fn, steps, stream, barrier=None, reduce=None, warm=3):
    """Mean µs per call of `steps` back-to-back calls between one event pair on `stream`."""
    import torch

    for _ in range(warm):
        fn()
    (barrier or torch.cuda.synchronize)()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(steps):
        fn()
    b.record(stream)
    b.synchronize()
    us = a.elapsed_time(b) / steps * 1e3
    return reduce(us) if reduce else us


def flushed_call_us(fn, y, L, device, stream, runs=20, warm=5):
    """The reference's timing protocol (applications/gemv/src/gemv_k1024_persistent_subwarp.cu:279-355):
    `warm` warm-up calls, then per call: y cleared, L2 flushed, a device sync, one event pair around
    the single launch; the mean over `runs`."""
    import torch

    for _ in range(warm):
        fn()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    total = 0.0
    for _ in range(runs):
        y.zero_()
        L.l2_flush(device, stream)
        torch.cuda.synchronize()
        a.record(stream)
        fn()
        b.record(stream)
        b.synchronize()
        total += a.elapsed_time(b)
    return total / runs * 1e3


def cublas_cli_us(M, N, dt, runs, warm, flush):
    """µs per call of the cuBLAS comparator binary (gemv_cublas_benchmark, the reference's cuBLAS
    column: one event pair per call, L2 flushed before each when flush=1)."""
    import subprocess

    exe = os.path.join(REPO, "l2domain_b200", "bin", "gemv_cublas_benchmark")
    try:
        r = subprocess.run([exe, str(M), str(N), str(runs), str(warm), str(flush), DT_NAME[dt]], capture_output=True,
                           text=True, timeout=300)
    except (OSError, subprocess.TimeoutExpired):
        return None
    for line in r.stdout.splitlines():
        t = line.split()
        if t and t[0] == "cublas_ms":
            return round(float(t[1]) * 1e3, 3)
    return None


def aligned_buffer(torch, dev, nbytes):
    raw = torch.empty(nbytes + (2 << 20), dtype=torch.uint8, device=dev)
    off = (-raw.data_ptr()) % (2 << 20)
    return raw, raw[off: off + nbytes]


def side_configs(L, torch, dev, local, stream, copy_peak, read_peak):
    """µs and GB/s per mode for configs 1-4 and the L2-window shape on this GPU, next to cuBLAS."""
    tdt = {F32: torch.float32, F16: torch.float16, BF16: torch.bfloat16}
    sink = torch.empty(4096, dtype=torch.int32, device=dev)
    out = {}

    def setup(M, N, dt, adist, xdist, batch=1):
        raw, A = aligned_buffer(torch, dev, batch * M * N * EB[dt])
        L.fill_cfg(A, dt, batch * M * N, 0, 0, *adist)
        x = torch.empty(batch * N * EB[dt], dtype=torch.uint8, device=dev)
        L.fill_cfg(x, dt, batch * N, 0, 1, *xdist)
        y = torch.empty(batch * M * EB[dt], dtype=torch.uint8, device=dev)
        plan = L.GemvPlan(A, M, N, dt, dt, batch=batch, device=local)
        return raw, A, x, y, plan

    def per_mode(plan, A, x, y, calls):
        return {name: round(kernel_time_us(lambda m=mode: plan.gemv(A, x, y, m, stream), calls, stream), 3)
                for name, mode in MODE_NAMES}

    def gbs(nbytes, us):
        return {k: round(nbytes / (v * 1e-6) / 1e9, 1) for k, v in us.items() if v}

    def sided_us(A, x, y, M, N, dt, calls, pooled=False):
        """The same matrix packed by L2 domain (l2d_sided_*; pooled: on pages of the domain-classified
        pool, l2d_sided_create_pooled): µs per call of each mode."""
        s = L.SidedMatrix(M, N, dt, dt, device=local, pooled=pooled)
        s.pack(A, stream=stream)
        res = {name: round(kernel_time_us(lambda m=mode: s.gemv(x, y, m, stream), calls, stream), 3)
               for name, mode in (("aware", 1), ("swapped", 2), ("stream", 3))}
        s.close()
        return res

    def other_placement(plan, A, x, y, M, N, dt, calls, batch=1):
        """The split modes under the placement the plan did not pick (granules <-> whole rows)."""
        mine = plan.stats()["placement"]
        other = "granules" if mine == 1 else "rows"
        p2 = L.GemvPlan(A, M, N, dt, dt, batch=batch, device=local, placement=other)
        res = {name: round(kernel_time_us(lambda m=mode: p2.gemv(A, x, y, m, stream), calls, stream), 3)
               for name, mode in MODE_NAMES if mode != 3}
        p2.close()
        return {"plan_placement": PLACEMENTS[mine], "other_placement": other, "us": res}

    def read_gbs(buf, nbytes, calls, passes=1):
        nb = nbytes // 32 * 32
        us = kernel_time_us(lambda: L.read_stream(buf, nb, sink, 4096, local, stream, passes=passes), calls, stream)
        return round(nb * passes / (us * 1e-6) / 1e9, 1)

    # Config 2: L2-resident fp16 4096x4096, 1000 back-to-back calls, against the L2 read peak.
    M, N, dt = 4096, 4096, F16
    raw, A, x, y, plan = setup(M, N, dt, (NORMAL, 0.0, 0.02), (NORMAL, 0.0, 1.0))
    nbytes = M * N * 2 + N * 2 + M * 2
    l2_peak = read_gbs(A, M * N * 2, 20, passes=50)  # 50 passes over the L2-resident 32 MiB per launch
    l2_launch = read_gbs(A, M * N * 2, 1000)          # one pass per launch: launch-bound like the GEMV
    us = per_mode(plan, A, x, y, 1000)
    A2, xv, yv = A.view(tdt[dt]).view(M, N), x.view(tdt[dt]), y.view(tdt[dt])
    us["cublas_torch_mv"] = round(kernel_time_us(lambda: torch.mv(A2, xv, out=yv), 1000, stream), 3)
    g = gbs(nbytes, us)
    out["cfg2"] = {"workload": "fp16 4096x4096 (32 MiB), 1000 back-to-back calls, no flush (L2-resident)",
                   "bound": "l2", "us": us, "gbs": g, "l2_read_peak_gbs": l2_peak,
                   "read_stream_one_pass_per_launch_gbs": l2_launch,
                   "frac_of_l2_read_peak": {k: round(v / l2_peak, 4) for k, v in g.items()},
                   "cublas_cli_us_per_event_pair": cublas_cli_us(M, N, dt, 200, 20, 0),
                   "sided_us": sided_us(A, x, y, M, N, dt, 1000),
                   "sided_pool_us": sided_us(A, x, y, M, N, dt, 1000, pooled=True),
                   "placements": other_placement(plan, A, x, y, M, N, dt, 1000)}
    plan.close()
    del raw, A

    # The L2 window: fp16 3584x16384 (112 MiB) fits in the two L2 halves only when each half keeps
    # its own domain's lines, so the near-domain split shows here.
    M, N, dt = 3584, 16384, F16
    raw, A, x, y, plan = setup(M, N, dt, (NORMAL, 0.0, 0.02), (NORMAL, 0.0, 1.0))
    us = per_mode(plan, A, x, y, 500)
    g = gbs(M * N * 2 + N * 2 + M * 2, us)
    out["l2_window"] = {"workload": "fp16 3584x16384 (112 MiB), 500 back-to-back calls, no flush", "bound": "l2",
                        "us": us, "gbs": g, "read_stream_gbs": read_gbs(A, M * N * 2, 500),
                        "read_stream_gbs_20_passes_per_launch": read_gbs(A, M * N * 2, 20, passes=20),
                        "aware_speedup_vs_stream": round(us["stream"] / us["aware"], 4),
                        "aware_speedup_vs_oblivious": round(us["oblivious"] / us["aware"], 4),
                        "swapped_slowdown_vs_aware": round(us["swapped"] / us["aware"], 4),
                        "sided_us": sided_us(A, x, y, M, N, dt, 500),
                   "sided_pool_us": sided_us(A, x, y, M, N, dt, 500, pooled=True),
                        "placements": other_placement(plan, A, x, y, M, N, dt, 500)}
    plan.close()
    del raw, A

    # Config 1: fp32 4096x4096 U[-1,1], the reference protocol (L2 flushed, one event pair per call)
    # and back to back (64 MiB stays in L2).
    M, N, dt = 4096, 4096, F32
    raw, A, x, y, plan = setup(M, N, dt, (UNIFORM, -1.0, 1.0), (UNIFORM, -1.0, 1.0))
    nbytes = M * N * 4 + N * 4 + M * 4
    A2, xv, yv = A.view(torch.float32).view(M, N), x.view(torch.float32), y.view(torch.float32)
    flushed = {name: round(flushed_call_us(lambda m=mode: plan.gemv(A, x, y, m, stream), y, L, local, stream), 3)
               for name, mode in MODE_NAMES}
    flushed["cublas_torch_mv"] = round(flushed_call_us(lambda: torch.mv(A2, xv, out=yv), y, L, local, stream), 3)
    flushed["cublas_cli"] = cublas_cli_us(M, N, dt, 20, 5, 1)
    steady = per_mode(plan, A, x, y, 200)
    steady["cublas_torch_mv"] = round(kernel_time_us(lambda: torch.mv(A2, xv, out=yv), 200, stream), 3)
    gf = gbs(nbytes, flushed)
    out["cfg1"] = {"workload": "fp32 4096x4096 (64 MiB), U[-1,1] seed 0",
                   "reference_protocol": {"protocol": "5 warm-ups, then per call: y cleared, L2 flushed, sync, one "
                                                      "event pair around the launch; mean of 20", "bound": "hbm",
                                          "us": flushed, "gbs": gf,
                                          "frac_of_read_peak": {k: round(v / read_peak, 4) for k, v in gf.items()}
                                          if read_peak else None},
                   "back_to_back": {"protocol": "200 back-to-back calls, no flush (64 MiB stays in L2)", "bound": "l2",
                                    "us": steady, "gbs": gbs(nbytes, steady),
                                    "placements": other_placement(plan, A, x, y, M, N, dt, 200)}}
    plan.close()
    del raw, A

    # Config 3: bf16 28672x8192 (448 MiB, larger than L2), 50 back-to-back calls.
    M, N, dt = 28672, 8192, BF16
    raw, A, x, y, plan = setup(M, N, dt, (NORMAL, 0.0, 0.02), (NORMAL, 0.0, 1.0))
    nbytes = M * N * 2 + N * 2 + M * 2
    us = per_mode(plan, A, x, y, 50)
    A2, xv, yv = A.view(torch.bfloat16).view(M, N), x.view(torch.bfloat16), y.view(torch.bfloat16)
    us["cublas_torch_mv"] = round(kernel_time_us(lambda: torch.mv(A2, xv, out=yv), 50, stream), 3)
    g = gbs(nbytes, us)
    out["cfg3"] = {"workload": "bf16 28672x8192 (448 MiB), 50 back-to-back calls (inputs larger than L2)",
                   "bound": "hbm", "us": us, "gbs": g,
                   "frac_of_read_peak": {k: round(v / read_peak, 4) for k, v in g.items()} if read_peak else None,
                   "frac_of_copy_peak": {k: round(v / copy_peak, 4) for k, v in g.items()},
                   "cublas_cli_us_per_event_pair": cublas_cli_us(M, N, dt, 20, 5, 0),
                   "sided_us": sided_us(A, x, y, M, N, dt, 50),
                   "sided_pool_us": sided_us(A, x, y, M, N, dt, 50, pooled=True),
                   "placements": other_placement(plan, A, x, y, M, N, dt, 50)}
    plan.close()
    del raw, A

    L.pool_release(local)  # the pooled sided matrices are gone: unmap the pool's chunks

    # Config 4: batched fp16 32 x (8192x8192) (4 GiB), 10 back-to-back calls.
    B, M, N, dt = 32, 8192, 8192, F16
    raw, A, x, y, plan = setup(M, N, dt, (UNIFORM, -0.05, 0.05), (NORMAL, 0.0, 1.0), batch=B)
    nbytes = B * (M * N * 2 + N * 2 + M * 2)
    us = per_mode(plan, A, x, y, 10)
    A3, x3, y3 = A.view(torch.float16).view(B, M, N), x.view(torch.float16).view(B, N, 1), \
        y.view(torch.float16).view(B, M, 1)
    us["cublas_torch_bmm"] = round(kernel_time_us(lambda: torch.bmm(A3, x3, out=y3), 10, stream), 3)
    g = gbs(nbytes, us)
    out["cfg4"] = {"workload": "fp16 32 x (8192x8192) contiguous batch (4 GiB), 10 back-to-back calls",
                   "bound": "hbm", "us": us, "gbs": g,
                   "frac_of_read_peak": {k: round(v / read_peak, 4) for k, v in g.items()} if read_peak else None,
                   "kernel": "ring (TMA bulk copies)" if plan.stats()["ring_modes"] & 2 else "register",
                   "placements": other_placement(plan, A, x, y, M, N, dt, 10, batch=B)}
    plan.close()
    del raw, A
    torch.cuda.empty_cache()
    return out


# ------------------------------------------------------------------------------------------------
# Our arm
# ------------------------------------------------------------------------------------------------

def cpu_baseline_leg(A_dev, x_dev, dt, N, budget_s):
    """The oracle's single-threaded CPU check loop on the first rows of the same matrix."""
    import torch

    import oracle as O
    rows = 1024
    st = torch.int16 if dt != F32 else torch.float32
    A = A_dev[: rows * N * EB[dt]].view(st).cpu().numpy()
    x = x_dev[: N * EB[dt]].view(st).cpu().numpy()
    if dt != F32:
        A, x = A.view(np.uint16), x.view(np.uint16)
    passes, t0 = 0, time.perf_counter()
    while True:
        O.gemv_seq(A, x, dt, rows, N)
        passes += 1
        el = time.perf_counter() - t0
        if el >= budget_s:
            break
    per = el / passes
    nbytes = rows * N * EB[dt] + N * EB[dt] + rows * EB[dt]
    return {"value": round(nbytes / per / 1e9, 4), "unit": "GB/s", "cores": 1, "kind": "port",
            "sample": f"rows 0..{rows - 1} ({rows}x{N} {DT_NAME[dt]}) of the same matrix, {passes} passes of the "
                      f"sequential fp32 check loop (gemv_k1024_persistent_subwarp.cu:383-390), 1 thread, "
                      f"{el:.1f} s"}


def run_ours(args, rank, world, local):
    import torch
    import torch.distributed as dist

    import l2domain_b200 as L

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    W = WORKLOADS[args.workload]
    M, N, batch, dt = W["M"], W["N"], W["batch"], W["dtype"]
    if args.rows:
        M = args.rows
    if batch != 1 and world > 1:
        raise SystemExit("batched workloads run on one GPU")
    if M % world:
        raise SystemExit(f"M={M} does not split over {world} ranks")
    m_loc = M // world
    eb = EB[dt]
    stream = torch.cuda.current_stream(dev)

    # A shard: 2 MiB aligned, generated on the device (rows [rank*m_loc, (rank+1)*m_loc) of the matrix).
    a_bytes = batch * m_loc * N * eb
    raw = torch.empty(a_bytes + (2 << 20), dtype=torch.uint8, device=dev)
    off = (-raw.data_ptr()) % (2 << 20)
    A = raw[off: off + a_bytes]
    L.fill_cfg(A, dt, batch * m_loc * N, 0, 0, *W["a"], first=rank * m_loc * N)
    x = torch.empty(batch * N * eb, dtype=torch.uint8, device=dev)
    if rank == 0:
        L.fill_cfg(x, dt, batch * N, 0, 1, *W["x"])
    else:
        x.zero_()
    y_loc = torch.empty(batch * m_loc * eb, dtype=torch.uint8, device=dev)
    y_full = torch.empty(batch * M * eb, dtype=torch.uint8, device=dev) if world > 1 else y_loc
    torch.cuda.synchronize()

    t_plan = time.perf_counter()
    plan = L.GemvPlan(A, m_loc, N, dt, dt, batch=batch, device=local,
                      tma={"auto": None, "ring": True, "register": False}[args.kernel])
    t_plan = time.perf_counter() - t_plan
    pstats = plan.stats()

    from l2domain_b200.shard import RowShard, ShardedGemvStep

    shard = RowShard(M, world, rank)
    assert shard.rows == m_loc and shard.row0 == rank * m_loc
    pstep = None
    if world > 1 and args.collective == "p2p":
        from l2domain_b200.shard import PeerGemvStep, exchange_bytes

        pstep = PeerGemvStep(shard, plan, N, dt, dt, local, lambda b: exchange_bytes(b, device=dev))
        if rank == 0:  # the step's input x, resident in both parities of rank 0's x buffer
            for par in (0, 1):
                pstep.x(par).copy_(x)
        torch.cuda.synchronize()

    def step(mode=L.MODE_AWARE, ev=None):
        if pstep is not None:
            if ev is not None:
                ev[0].record(stream)
            par = pstep(mode, stream)
            if ev is not None:
                ev[1].record(stream)
            return par

        def local():
            if ev is not None:
                ev[0].record(stream)
            plan.gemv(A, x, y_loc, mode, stream)
            if ev is not None:
                ev[1].record(stream)

        ShardedGemvStep(shard, x, y_loc, y_full, local)()

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])
        torch.cuda.synchronize()

    def max_over_ranks(v: float) -> float:
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # Sanity check against a float64 torch dot product on sampled rows (the oracle is not used here).
    ShardedGemvStep(shard, x, y_loc, y_full, lambda: plan.gemv(A, x, y_loc, L.MODE_AWARE, stream))()
    torch.cuda.synchronize()
    gather_exact = None
    if pstep is not None:  # the peer-memory gather must equal the NCCL gather bit for bit
        par = step()
        torch.cuda.synchronize()
        gather_exact = bool(torch.equal(pstep.y(par), y_full))
        if not gather_exact or pstep.status():
            raise SystemExit(f"rank {rank}: peer-memory step differs from NCCL (status {pstep.status()})")
    tdt = {F32: torch.float32, F16: torch.float16, BF16: torch.bfloat16}[dt]
    Av = A.view(tdt).view(batch * m_loc, N)
    xv = x.view(tdt)
    idx = torch.linspace(0, batch * m_loc - 1, 64, device=dev).long()
    bidx = idx // m_loc
    ref = (Av[idx].double() * xv.view(batch, N)[bidx].double()).sum(1)
    got = y_loc.view(tdt)[idx].double()
    # Every rank checks 64 rows of its own shard; with the gathered y equal to the NCCL gather of the
    # shards, that covers sampled rows of every rank's part of y.  The worst rank is reported.
    rel = max_over_ranks(float(((got - ref).norm() / ref.norm()).item()))
    if not rel <= 2e-3:
        raise SystemExit(f"rank {rank}: GEMV self-check failed, rel L2 {rel:.3g} (worst rank)")

    # Headline: K timed steps of the aware GEMV (plus the exchange at N > 1).  The clock sampler
    # starts before the warm-up so its thread and NVML are warm when the timed region begins.
    sampler = ClockSampler(local).start()
    for _ in range(args.warmup):
        step()
    barrier()
    # When a step is one GEMV launch (N=1, or the peer-memory exchange fused into it), the kernel's
    # average launch duration is the loop time over K, and no event sits between two launches: an
    # event there would keep each launch from overlapping the previous one's tail (programmatic
    # dependent launch).  With NCCL collectives in the step, events bracket each GEMV launch.
    one_launch = world == 1 or pstep is not None
    kev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with sampler:
        e0.record(stream)
        for i in range(args.steps):
            step(L.MODE_AWARE, None if one_launch else kev[i])
        e1.record(stream)
        e1.synchronize()
    barrier()
    step_ms = max_over_ranks(e0.elapsed_time(e1) / args.steps)
    if one_launch:
        kern_ms = step_ms
    else:
        kern_ms = max_over_ranks(sum(a.elapsed_time(b) for a, b in kev) / args.steps)

    bytes_loc = a_bytes + batch * N * eb + batch * m_loc * eb
    total_bytes = bytes_loc * world
    value = total_bytes / (step_ms * 1e-3) / 1e9
    peak, peak_src = measured_peaks()
    achieved = bytes_loc / (kern_ms * 1e-3) / 1e9
    traffic = profiled_traffic(args.workload, batch * m_loc)

    # Per-mode kernel times on the same data (the domain effect), and the cuBLAS comparator.
    modes_us = {}
    if not args.no_aux:
        def kernel_time(fn, steps):
            return kernel_time_us(fn, steps, stream, barrier, max_over_ranks)

        for name, mode in MODE_NAMES:
            modes_us[name] = round(kernel_time(lambda m=mode: plan.gemv(A, x, y_loc, m, stream), args.steps), 3)
        if batch == 1:
            out = torch.empty(m_loc, dtype=tdt, device=dev)
            A2 = A.view(tdt).view(m_loc, N)
            modes_us["cublas_torch_mv"] = round(kernel_time(lambda: torch.mv(A2, xv, out=out), args.steps), 3)
        Ai = A.view(torch.int64)
        modes_us["torch_sum_read"] = round(kernel_time(lambda: torch.sum(Ai), max(5, args.steps // 5)), 3)

    # Read-only stream over this rank's A (larger than L2): the HBM read bandwidth of this box, the
    # denominator beside the copy peak for a read-dominated kernel.
    read_peak = None
    if not args.no_aux:
        sink = torch.empty(4096, dtype=torch.int32, device=dev)
        rb = a_bytes // 32 * 32
        read_us = kernel_time_us(lambda: L.read_stream(A, rb, sink, 4096, local, stream), max(5, args.steps // 5),
                                 stream, barrier, max_over_ranks)
        read_peak = round(rb / (read_us * 1e-6) / 1e9, 1)

    # Side measurements of the other BASELINE configs (N=1 only): not the headline.
    configs = None
    if not args.no_aux and world == 1:
        configs = side_configs(L, torch, dev, local, stream, peak, read_peak)

    # End to end through the public API: pinned x in, y out, every step.
    x_host = torch.empty_like(x, device="cpu").pin_memory()
    x_host.copy_(x)
    y_host = torch.empty_like(y_full, device="cpu").pin_memory()

    def e2e_step():
        if pstep is not None:
            par = pstep.next_parity()
            if rank == 0:
                pstep.x(par).copy_(x_host, non_blocking=True)
            step()
            y_host.copy_(pstep.y(par), non_blocking=True)
            return
        if rank == 0:
            x.copy_(x_host, non_blocking=True)
        step()
        y_host.copy_(y_full, non_blocking=True)

    for _ in range(args.warmup):
        e2e_step()
    barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(args.steps):
        e2e_step()
    b.record(stream)
    b.synchronize()
    e2e_ms = max_over_ranks(a.elapsed_time(b) / args.steps)
    barrier()
    fstats = plan.stats()

    cpu = None
    if rank == 0 and world == 1:
        cpu = cpu_baseline_leg(A, x, dt, N, args.cpu_seconds)

    if rank == 0:
        clocks = sampler.summary()
        exchange = (", peer-memory x push + y gather inside the GEMV launch (CUDA IPC over NVLink)"
                    if pstep is not None else ", NCCL broadcast(x) + all_gather(y)")
        ratio = None
        if modes_us.get("oblivious") and modes_us.get("aware"):
            ratio = round(modes_us["oblivious"] / modes_us["aware"], 4)
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(step_ms, 6), "us_per_call": round(step_ms * 1e3, 3),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": DT_NAME[dt],
            "data": "synthetic: seeded splitmix64 stream, A~N(0,0.02), x~N(0,1) (cfg5 distributions), generated on device",
            "config": {"workload": f"{args.workload}: {W['name']}", "M": M, "N": N, "batch": batch,
                       "dtype_in": DT_NAME[dt], "dtype_out": DT_NAME[dt], "rows_per_gpu": m_loc,
                       "parallelism": f"row-shard x{world}" + (exchange if world > 1 else ""),
                       "mode": "aware", "l2": f"inputs larger than L2 ({a_bytes / 2**20:.0f} MiB of A per GPU), no flush"},
            "modes_us": modes_us, "aware_speedup_vs_oblivious": ratio, "configs": configs,
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "traffic": traffic, "peak_source": peak_src,
                         "read_peak": read_peak,
                         "read_peak_source": "measured in this run: l2d_read_stream over this rank's A, back to back",
                         "frac_of_read_peak": round(achieved / read_peak, 4) if read_peak else None,
                         "frac_of_spec_8TBs": round(achieved / SPEC_HBM_GBS, 4), "kernel_us": round(kern_ms * 1e3, 3),
                         "bytes_per_launch": bytes_loc},
            "cpu_baseline": cpu,
            "e2e": {"value": round(total_bytes / (e2e_ms * 1e-3) / 1e9, 2), "unit": "GB/s",
                    "h2d_bytes_per_step": int(x.numel()), "d2h_bytes_per_step": int(y_full.numel()),
                    "ms_per_step": round(e2e_ms, 6)},
            "gpu_launches": args.steps,
            "clocks": clocks,
            "plan": {"probe_and_plan_s": round(t_plan, 3), "domain_sms": pstats["domain_sms"],
                     "granule_shift": pstats["granule_shift"], "domain_bytes": pstats["domain_bytes"],
                     "split_rows": pstats["split_rows"], "fallback_slots": fstats["fallback_slots"],
                     "calls": fstats["calls"], "placement": PLACEMENTS[pstats["placement"]],
                     "kernel": "ring (TMA bulk copies)" if fstats["ring_modes"] & (1 << L.MODE_AWARE) else "register"},
            "check": {"rows_per_rank": 64, "rel_l2_vs_torch_f64_worst_rank": rel,
                      "p2p_gather_equals_nccl": gather_exact},
        }
        print(json.dumps(line), flush=True)
    if pstep is not None:
        barrier()
        pstep.close()
    plan.close()
    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()
    return 0


def main():
    args = parse()
    rank, world, local = dist_env()
    if args.gpus != world and world != 1:
        print(f"warning: --gpus {args.gpus} but WORLD_SIZE {world}", file=sys.stderr)
    if args.impl == "reference":
        return run_reference(args, rank, world)
    return run_ours(args, rank, world, local)


if __name__ == "__main__":
    sys.exit(main())
