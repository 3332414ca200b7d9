"""The run.sh drop-in and its binaries: CPU-side option handling and dry runs, plus (GPU) the
process contract the reference's runner parses (applications/gemv/run.sh:62-98)."""
import csv
import json
import os
import subprocess

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
RUN = os.path.join(REPO, "l2domain_b200", "gemv", "run.sh")
BIN = os.path.join(REPO, "l2domain_b200", "bin")
PLOT = os.path.join(REPO, "l2domain_b200", "gemv", "plot_gemv.py")


def sh(*args, env=None, timeout=600):
    return subprocess.run(["bash", RUN, *args], capture_output=True, text=True, env=env, timeout=timeout)


def test_dry_run_quick_prints_reference_commands():
    r = sh("--dry-run", "--preset", "quick")
    assert r.returncode == 0, r.stderr
    assert "gemv_sidegpu_l32_w16 2048 5 4242 1 1024 fp32" in r.stdout
    assert "gemv_cublas_benchmark 2048 1024 5 1 1 fp32" in r.stdout


def test_dry_run_paper_sweep():
    r = sh("--dry-run", "--preset", "paper", "--dtype", "bf16", "--k", "4096")
    assert r.returncode == 0, r.stderr
    for m in range(2048, 10241, 1024):
        assert f"gemv_sidegpu_l32_w16 {m} 50 4242 1 4096 bf16" in r.stdout
        assert f"gemv_cublas_benchmark {m} 4096 20 5 1 bf16" in r.stdout


@pytest.mark.parametrize("args", [["--preset", "full"], ["--device", "x"], ["--wait-timeout", "-1"],
                                  ["--arch", "sm_90a"], ["--dtype", "fp8"], ["--bogus"], ["--preset"]])
def test_bad_options_exit_2(args):
    assert sh(*args, "--dry-run").returncode == 2


def write_csv(path, rows):
    cols = ["M", "K", "lanes_per_row", "warps_per_block", "baseline_ms", "aware_ms", "swapped_ms", "cublas_ms",
            "max_abs_error", "aware_speedup", "swapped_speedup", "aware_vs_cublas", "pass", "dtype", "aware_gbs"]
    with open(path, "w") as f:
        w = csv.writer(f)
        w.writerow(cols)
        for r in rows:
            w.writerow(r)


def row(m=2048, k=1024, p="PASS"):
    return [m, k, 32, 16, 0.01, 0.009, 0.011, 0.012, 1e-6, 1.1, 0.9, 1.3, p, "fp32", 900.0]


def test_plot_gate_accepts_and_refuses(tmp_path):
    write_csv(tmp_path / "final_gemv_B200.csv", [row(), row(3072)])
    assert subprocess.run(["python3", PLOT, "--data-dir", str(tmp_path), "--output-dir", str(tmp_path)]).returncode == 0
    write_csv(tmp_path / "final_gemv_B200.csv", [row(), row(3072, p="FAIL")])
    assert subprocess.run(["python3", PLOT, "--data-dir", str(tmp_path), "--output-dir", str(tmp_path)],
                          capture_output=True).returncode != 0
    write_csv(tmp_path / "final_gemv_B200.csv", [row(), row(3072, k=2048)])
    assert subprocess.run(["python3", PLOT, "--data-dir", str(tmp_path), "--output-dir", str(tmp_path)],
                          capture_output=True).returncode != 0


def parse(out, key):
    for line in out.splitlines():
        t = line.split()
        if t and t[0] == key:
            return float(t[1])
    return None


@pytest.mark.gpu
def test_binary_contract_quick(tmp_path):
    pytest.importorskip("torch").cuda.is_available() or pytest.skip("no GPU")
    env = dict(os.environ, SIDEDGPU_CONFIG_DIR=str(tmp_path))
    r = subprocess.run([os.path.join(BIN, "gemv_sidegpu_l32_w16"), "2048", "3", "4242", "1"], capture_output=True,
                       text=True, env=env, timeout=300)
    assert r.returncode == 0, r.stderr
    for key in ("baseline_ms", "aware_ms", "swapped_ms"):
        assert parse(r.stdout, key) > 0
    line = [l for l in r.stdout.splitlines() if "correctness max_abs_error" in l][0]
    errs = [float(t.split("=")[1]) for t in line.split() if "=" in t]
    assert len(errs) == 3 and max(errs) <= 1e-3
    assert open(tmp_path / "smid2side.csv").read().count(",") >= 100
    assert open(tmp_path / "mask.csv").read().startswith("0x")
    c = subprocess.run([os.path.join(BIN, "gemv_cublas_benchmark"), "2048", "1024", "3", "1", "1"],
                       capture_output=True, text=True, timeout=300)
    assert c.returncode == 0, c.stderr
    assert parse(c.stdout, "cublas_ms") > 0


@pytest.mark.gpu
@pytest.mark.parametrize("dtype,M,K", [("fp16", 4096, 4096), ("bf16", 28672, 8192), ("fp32", 4096, 4096)])
def test_cublas_comparator_dtypes(dtype, M, K):
    """The cuBLAS column at the new dtypes (cublasGemmEx with fp32 compute for fp16/bf16; the
    reference's binary has only cublasSgemv, gemv_cublas_benchmark.cu:75-89): same argv and stdout
    contract, a positive time, and the matrix size it reports matches the dtype."""
    pytest.importorskip("torch").cuda.is_available() or pytest.skip("no GPU")
    c = subprocess.run([os.path.join(BIN, "gemv_cublas_benchmark"), str(M), str(K), "5", "2", "0", dtype],
                       capture_output=True, text=True, timeout=300)
    assert c.returncode == 0, c.stderr
    assert parse(c.stdout, "cublas_ms") > 0
    eb = 4 if dtype == "fp32" else 2
    assert f"matrix={M * K * eb / 2**20:.1f} MiB" in c.stdout
    assert ("SGEMV" in c.stdout) == (dtype == "fp32")


@pytest.mark.gpu
def test_calibration_tools(tmp_path):
    pytest.importorskip("torch").cuda.is_available() or pytest.skip("no GPU")
    env = dict(os.environ, SIDEDGPU_CONFIG_DIR=str(tmp_path))
    a = subprocess.run([os.path.join(BIN, "get_smid2side")], capture_output=True, text=True, env=env, timeout=120)
    assert a.returncode == 0, a.stderr
    b = subprocess.run([os.path.join(BIN, "get_mask")], capture_output=True, text=True, env=env, timeout=120)
    assert b.returncode == 0, b.stderr
    assert "mask = 0x" in b.stdout


PLAN_Y = r"""
import sys, json, torch
sys.path.insert(0, {repo!r})
import l2domain_b200 as L
torch.cuda.set_device(0)
M, N = 2048, 8192
raw = torch.empty(M * N * 2 + (2 << 20), dtype=torch.uint8, device="cuda")
off = (-raw.data_ptr()) % (2 << 20)
A = raw[off: off + M * N * 2]
L.fill_cfg(A, L.F16, M * N, 4, 0, 1, 0.0, 0.02)
x = torch.empty(N * 2, dtype=torch.uint8, device="cuda")
L.fill_cfg(x, L.F16, N, 4, 1, 1, 0.0, 1.0)
y = torch.empty(M * 2, dtype=torch.uint8, device="cuda")
plan = L.GemvPlan(A, M, N, L.F16, L.F16)
plan.gemv(A, x, y, L.MODE_AWARE)
torch.cuda.synchronize()
print(json.dumps({{"cached": plan.stats()["sm_map_cached"], "y": y.cpu().tolist()[:4096:7]}}))
"""


@pytest.mark.gpu
def test_domain_map_cache_reused_by_plans(tmp_path):
    """get_smid2side writes the map with its device key; --validate re-probes and agrees; a plan made
    in a fresh process with SIDEDGPU_CONFIG_DIR set reads the map instead of probing and gives the
    same bits as a probed plan; a cache keyed to another device is not used (the plan probes) and
    --validate reports it."""
    pytest.importorskip("torch").cuda.is_available() or pytest.skip("no GPU")
    env = dict(os.environ, SIDEDGPU_CONFIG_DIR=str(tmp_path))
    a = subprocess.run([os.path.join(BIN, "get_smid2side")], capture_output=True, text=True, env=env, timeout=120)
    assert a.returncode == 0, a.stderr
    assert (tmp_path / "l2d_device.txt").read_text().startswith("uuid=GPU-")
    v = subprocess.run([os.path.join(BIN, "get_smid2side"), "--validate"], capture_output=True, text=True, env=env,
                       timeout=120)
    assert v.returncode == 0 and "0 of" in v.stdout, v.stdout + v.stderr
    code = PLAN_Y.format(repo=REPO)
    run = lambda e: json.loads(subprocess.run(["python3", "-c", code], capture_output=True, text=True, env=e,
                                              timeout=300, check=True).stdout.strip().splitlines()[-1])
    plain = {k: v for k, v in os.environ.items() if k != "SIDEDGPU_CONFIG_DIR"}
    cached, probed = run(env), run(plain)
    assert cached["cached"] == 1 and probed["cached"] == 0
    assert cached["y"] == probed["y"]
    (tmp_path / "l2d_device.txt").write_text("uuid=GPU-another;sm=148\n")
    assert run(env)["cached"] == 0
    v = subprocess.run([os.path.join(BIN, "get_smid2side"), "--validate"], capture_output=True, text=True, env=env,
                       timeout=120)
    assert v.returncode == 4


@pytest.mark.gpu
def test_run_sh_quick_end_to_end(tmp_path):
    pytest.importorskip("torch").cuda.is_available() or pytest.skip("no GPU")
    r = sh("--preset", "quick", "--output-dir", str(tmp_path), "--wait-timeout", "60", timeout=900)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    rows = list(csv.DictReader(open(next(tmp_path.glob("final_gemv_*.csv")))))
    assert rows and all(x["pass"] == "PASS" for x in rows)
