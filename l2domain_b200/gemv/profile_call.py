"""One GEMV configuration, a few calls, for profiling with ncu (or timing a single shape).

    python -m l2domain_b200.gemv.profile_call --mib 32 --n 4096 --dtype fp16 --mode aware --warmup 5
        [--layout dense|sided|sharded] [--kernel auto|ring|register] [--placement auto|granules|rows]
        [--batch 1] [--calls 1]

Builds a synthetic A of about `mib` MiB with rows of `n` elements (A ~ N(0, 0.02), x ~ N(0, 1),
seed 0; `batch` problems of that size back to back), plans it (which runs the SM and address
probes once), then makes `warmup` calls and
`calls` more of one mode, so a capture can skip the warm-up launches (ncu -k regex:k_gemv -s W).
Layouts: the dense plan (l2d_gemv), the same matrix packed by L2 domain (l2d_gemv_sided), or a
one-rank peer-memory shard (l2d_gemv_sharded, the kernels the multi-GPU step runs).  Prints the mean
µs per call of the last `calls` calls (CUDA events; meaningless under a profiler).
"""
from __future__ import annotations

import argparse
import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

import l2domain_b200 as L  # noqa: E402


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--mib", type=int, default=32)
    ap.add_argument("--n", type=int, default=4096)
    ap.add_argument("--dtype", choices=sorted(L.DTYPES), default="fp16")
    ap.add_argument("--mode", choices=["aware", "oblivious", "swapped", "stream"], default="aware")
    ap.add_argument("--layout", choices=["dense", "sided", "sharded"], default="dense")
    ap.add_argument("--kernel", choices=["auto", "ring", "register"], default="auto")
    ap.add_argument("--placement", choices=["auto", "granules", "rows"], default="auto")
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--calls", type=int, default=1)
    args = ap.parse_args()

    import torch

    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    dt = L.DTYPES[args.dtype]
    eb = L.ELEM_BYTES[dt]
    N = args.n
    M = max(1, args.mib * 2**20 // (N * eb))
    B = max(1, args.batch)
    nb = B * M * N * eb
    raw = torch.empty(nb + (2 << 20), dtype=torch.uint8, device=dev)
    off = (-raw.data_ptr()) % (2 << 20)
    A = raw[off: off + nb]
    L.fill_cfg(A, dt, B * M * N, 0, 0, 1, 0.0, 0.02)
    x = torch.empty(B * N * eb, dtype=torch.uint8, device=dev)
    L.fill_cfg(x, dt, B * N, 0, 1, 1, 0.0, 1.0)
    y = torch.empty(B * M * eb, dtype=torch.uint8, device=dev)
    tma = {"auto": None, "ring": True, "register": False}[args.kernel]
    if B > 1 and args.layout != "dense":
        raise SystemExit("--batch applies to the dense layout")
    mode = L.MODES[args.mode]
    closers = []
    if args.layout == "dense":
        plan = L.GemvPlan(A, M, N, dt, dt, batch=B, tma=tma,
                          placement=None if args.placement == "auto" else args.placement)
        closers.append(plan)
        call = lambda: plan.gemv(A, x, y, mode)  # noqa: E731
    elif args.layout == "sided":
        s = L.SidedMatrix(M, N, dt, dt)
        s.pack(A)
        closers.append(s)
        call = lambda: s.gemv(x, y, mode)  # noqa: E731
    else:
        plan = L.GemvPlan(A, M, N, dt, dt, placement=None if args.placement == "auto" else args.placement)
        sh = L.PeerShard(0, 0, 1, M, 0, M, N, dt, dt)
        sh.connect([sh.handle()])
        for par in (0, 1):
            sh.x_tensor(par).copy_(x)
        closers += [sh, plan]
        call = lambda: sh.step(plan, mode)  # noqa: E731
    for _ in range(args.warmup):
        call()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(args.calls):
        call()
    b.record()
    b.synchronize()
    us = a.elapsed_time(b) / args.calls * 1e3
    for c in closers:
        c.close()
    print(json.dumps({"M": M, "N": N, "batch": B, "dtype": args.dtype, "mode": args.mode, "layout": args.layout,
                      "kernel": args.kernel, "placement": args.placement, "bytes": nb, "us_per_call": round(us, 3)}))
    return 0


if __name__ == "__main__":
    sys.exit(main())
