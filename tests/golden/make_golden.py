#!/usr/bin/env python3
"""Regenerate tests/golden/reference_pins.json from the reference itself.

Run where the reference tree is present (L2D_REFERENCE_ROOT, else a `reference` directory beside
this repository):

    make -C oracle ref            # compiles the reference's GEMV source in place -> oracle/_ref/
    python tests/golden/make_golden.py

What is pinned, and from where:
  * mix32 outputs           -- the reference's own `mix32` (gemv_k1024_persistent_subwarp.cu:56-63),
                               called through oracle/_ref/libref_pin.so.
  * reference-mode inputs   -- A/x values of the quick case built from the reference `mix32` and the
                               init_data formulas (gemv_k1024_persistent_subwarp.cu:118-139).
  * integer-input KAT       -- the reference's -DINTEGER_FLOAT_INPUTS mode (same file :122-134):
                               y computed in exact integer arithmetic, so any fp32 summation order
                               must reproduce it bit for bit.
  * predictor / partition   -- `predict_addr_side` (:105-108) and `predict_map_memory_attr_far`
                               (latopt.cuh:255-263) evaluated by the reference code on the H100 mask.
  * H100 latency fixtures   -- architecture/data/figure_04.csv (MaskProbe curves, mask 0xb3000) and
                               figure_05.csv (leader/follower trace), the only measured data the
                               reference ships for the domain probes.
The output is small JSON; the GPU box never needs the reference tree.
"""
from __future__ import annotations

import csv
import ctypes as C
import json
import os
import subprocess
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
REF = os.environ.get("L2D_REFERENCE_ROOT") or os.path.join(os.path.dirname(REPO), "reference")
PIN = os.path.join(REPO, "oracle", "_ref", "libref_pin.so")
OUT = os.path.join(HERE, "reference_pins.json")

H100_MASK = 0xB3000
GRAN = 2 * 1024 * 1024


def load_pin() -> C.CDLL:
    if not os.path.exists(PIN):
        subprocess.run(["make", "-s", "-C", os.path.join(REPO, "oracle"), "ref", f"REF={REF}"], check=True)
    L = C.CDLL(PIN)
    L.ref_mix32.restype = C.c_uint32
    L.ref_mix32.argtypes = [C.c_uint32]
    L.ref_predict_far.restype = C.c_int
    L.ref_predict_far.argtypes = [C.c_int, C.c_uint32, C.c_uint64, C.c_int]
    L.ref_predict_addr_side.restype = C.c_int
    L.ref_predict_addr_side.argtypes = [C.c_uint64, C.c_uint32, C.c_void_p, C.c_size_t, C.c_uint64]
    L.ref_memory_alloc_gran.restype = C.c_size_t
    return L


def main() -> int:
    L = load_pin()
    assert L.ref_memory_alloc_gran() == GRAN
    rng = np.random.default_rng(20261201)
    out: dict = {"generator": "tests/golden/make_golden.py", "reference_root_layout": "LyleLuo/L2Domain"}

    # mix32 on structured and random inputs.
    inputs = list(range(0, 512)) + [int(v) for v in rng.integers(0, 2**32, 512, dtype=np.uint64)]
    inputs += [0xFFFFFFFF, 0x80000000, 4242, 4242 + 0x9E37]
    out["mix32"] = {"in": inputs, "out": [int(L.ref_mix32(v)) for v in inputs]}

    # Reference-mode quick-case inputs (seed 4242, K=1024) at sampled flat indices.
    seed = 4242
    K = 1024
    idx = sorted(set([0, 1, 2, 1023, 1024, 2**20, 2**21 - 1] + [int(v) for v in rng.integers(0, 2048 * K, 200)]))
    a_vals, a_int = [], []
    for i in idx:
        h = L.ref_mix32((i & 0xFFFFFFFF) ^ seed)
        a_vals.append(float(np.float32(np.float32(h & 0xFF) / np.float32(255.0)) - np.float32(0.5)))
        a_int.append(int(h % 17) - 8)
    xs = list(range(K))
    x_vals, x_int = [], []
    for i in xs:
        h = L.ref_mix32((i ^ ((seed + 0x9E37) & 0xFFFFFFFF)) & 0xFFFFFFFF)
        x_vals.append(float(np.float32(np.float32(h & 0xFF) / np.float32(255.0)) - np.float32(0.5)))
        x_int.append(int(h % 7) - 3)
    out["ref_inputs"] = {"seed": seed, "K": K, "a_index": idx, "a": a_vals, "a_integer": a_int,
                         "x": x_vals, "x_integer": x_int}

    # Integer-input KAT: M = 1024 (the reference's minimum M), K = 1024, exact integer y.
    M = 1024
    flat = np.arange(M * K, dtype=np.uint64)
    hA = np.array([L.ref_mix32(int(v) ^ seed) for v in flat], dtype=np.uint64)
    Aint = (hA % 17).astype(np.int64) - 8
    xint = np.array(x_int, dtype=np.int64)
    y = Aint.reshape(M, K) @ xint
    out["integer_kat"] = {"seed": seed, "M": M, "K": K, "y": [int(v) for v in y],
                          "a_checksum": int(Aint.sum()), "a_abs_checksum": int(np.abs(Aint).sum())}

    # Predictor and partition on the H100 mask (2 MiB pages with a fixed attr pattern).
    base = 0x7F3A00000000  # 2 MiB aligned
    attr = [int(v) for v in rng.integers(0, 2, 16)]
    attr_arr = np.array(attr, dtype=np.int32)
    addrs = [base + int(v) * 128 for v in rng.integers(0, (16 * GRAN) // 128, 600)]
    sides = [int(L.ref_predict_addr_side(base, H100_MASK, attr_arr.ctypes.data, attr_arr.size, a)) for a in addrs]
    far_cases = []
    for _ in range(300):
        s = int(rng.integers(0, 2))
        m = int(rng.integers(0, 2**32, dtype=np.uint64))
        a = int(rng.integers(0, 2**48, dtype=np.uint64))
        t = int(rng.integers(0, 2))
        far_cases.append([s, m, a, t, int(L.ref_predict_far(s, m, a, t))])
    rows_M, row_bytes = 8192, 4096  # K=1024 fp32 rows, 32 MiB over 16 pages
    side0 = [r for r in range(rows_M)
             if L.ref_predict_addr_side(base, H100_MASK, attr_arr.ctypes.data, attr_arr.size, base + r * row_bytes) == 0]
    out["predictor"] = {"base": base, "mask": H100_MASK, "attr": attr, "addr": addrs, "side": sides,
                        "far_cases": far_cases}
    out["partition"] = {"base": base, "mask": H100_MASK, "attr": attr, "M": rows_M, "row_bytes": row_bytes,
                        "side0_rows": side0}

    # H100 probe fixtures shipped by the reference.
    f4 = os.path.join(REF, "architecture", "data", "figure_04.csv")
    with open(f4) as f:
        rows = list(csv.DictReader(f))
    out["h100_maskprobe"] = {
        "source": "architecture/data/figure_04.csv",
        "bit": [int(r["address_bit"]) for r in rows],
        "a_follower": [float(r["sm_a_follower_cycles"]) for r in rows],
        "b_follower": [float(r["sm_b_follower_cycles"]) for r in rows],
        "active": [int(r["active"]) for r in rows],
        "mask": H100_MASK,
    }
    f5 = os.path.join(REF, "architecture", "data", "figure_05.csv")
    with open(f5) as f:
        rows = list(csv.DictReader(f))
    out["h100_trace"] = {
        "source": "architecture/data/figure_05.csv",
        "round": [int(r["round_id"]) for r in rows],
        "offset": [int(r["offset_bytes"]) for r in rows],
        "latency": [int(r["latency_cycles"]) for r in rows],
        "mask": int(rows[0]["active_mask_hex"], 16),
    }
    with open(OUT, "w") as f:
        json.dump(out, f, separators=(",", ":"))
    print(f"wrote {OUT} ({os.path.getsize(OUT)} bytes)")
    return 0


if __name__ == "__main__":
    sys.exit(main())
