#!/usr/bin/env bash
# Drop-in for the reference's applications/gemv/run.sh: same options, presets, binaries, stdout
# parsing and CSV columns (M,K,...,pass), with trailing columns for the B200 extensions.
#
#   ./run.sh [--device auto|IDX|UUID] [--preset quick|paper] [--build-only] [--dry-run]
#            [--arch auto|sm_XX] [--wait-timeout S] [--poll-interval S] [--output-dir PATH]
#            [--dtype fp32|fp16|bf16] [--k N]
#
# quick: M=2048, 5 runs (cuBLAS 5 runs, 1 warm-up); paper: M=2048..10240 step 1024, 50/20/5.
# A case passes when both binaries exit 0, every time is positive and max_abs_error <= 1e-3
# (fp32; 2e-2 for fp16/bf16 inputs, whose products carry input rounding), as run.sh:94-97.
set -euo pipefail

APP_DIR="$(cd "$(dirname "${BASH_SOURCE[0]}")" && pwd)"
PKG_DIR="$(cd "${APP_DIR}/.." && pwd)"

DEVICE=auto PRESET=quick BUILD_ONLY=0 DRY_RUN=0 ARCH=auto WAIT_TIMEOUT=1800 POLL_INTERVAL=10
OUTPUT_ARG=out DTYPE=fp32 K=1024

usage() {
  cat <<'USAGE'
Usage: ./run.sh [common options]

  --device auto|INDEX|UUID  GPU selection (default: auto)
  --preset quick|paper     Smoke point or paper sweep (default: quick)
  --dtype fp32|fp16|bf16   Input/output type (default: fp32, the reference's)
  --k N                    Row length K (default: 1024, the reference's)
  --build-only             Compile without running
  --dry-run                Print commands without executing them
  --arch auto|sm_XX        Override CUDA architecture detection (only sm_100a is built)
  --wait-timeout SECONDS   Wait for a free GPU (default: 1800)
  --poll-interval SECONDS  GPU polling interval (default: 10)
  --output-dir PATH        Runtime output directory (default: out)
USAGE
}

need() { if (( $# < 2 )); then echo "missing value for $1" >&2; exit 2; fi; }
while (( $# > 0 )); do
  case "$1" in
    --device) need "$@"; DEVICE="$2"; shift 2 ;;
    --preset) need "$@"; PRESET="$2"; shift 2 ;;
    --build-only) BUILD_ONLY=1; shift ;;
    --dry-run) DRY_RUN=1; shift ;;
    --arch) need "$@"; ARCH="$2"; shift 2 ;;
    --wait-timeout) need "$@"; WAIT_TIMEOUT="$2"; shift 2 ;;
    --poll-interval) need "$@"; POLL_INTERVAL="$2"; shift 2 ;;
    --output-dir) need "$@"; OUTPUT_ARG="$2"; shift 2 ;;
    --dtype) need "$@"; DTYPE="$2"; shift 2 ;;
    --k) need "$@"; K="$2"; shift 2 ;;
    -h|--help) usage; exit 0 ;;
    *) echo "unknown option: $1" >&2; usage >&2; exit 2 ;;
  esac
done

[[ "${WAIT_TIMEOUT}" =~ ^[0-9]+$ ]] || { echo "--wait-timeout must be a non-negative integer" >&2; exit 2; }
[[ "${POLL_INTERVAL}" =~ ^[0-9]+$ ]] || { echo "--poll-interval must be a non-negative integer" >&2; exit 2; }
[[ "${DEVICE}" == auto || "${DEVICE}" =~ ^[0-9]+$ || "${DEVICE}" =~ ^GPU-[A-Za-z0-9-]+$ ]] \
  || { echo "--device must be auto, a physical GPU index, or a full GPU UUID" >&2; exit 2; }
[[ "${ARCH}" == auto || "${ARCH}" =~ ^(sm_)?100a?$ ]] \
  || { echo "this build targets sm_100a only (got --arch ${ARCH})" >&2; exit 2; }
[[ "${DTYPE}" =~ ^(fp32|fp16|bf16)$ ]] || { echo "--dtype must be fp32, fp16 or bf16" >&2; exit 2; }
[[ "${K}" =~ ^[0-9]+$ && "${K}" -gt 0 ]] || { echo "--k must be a positive integer" >&2; exit 2; }
[[ -n "${OUTPUT_ARG}" ]] || { echo "--output-dir must not be empty" >&2; exit 2; }

case "${PRESET}" in
  quick) M_VALUES="2048"; OUR_RUNS=5; CUBLAS_RUNS=5; WARMUPS=1 ;;
  paper) M_VALUES="2048 3072 4096 5120 6144 7168 8192 9216 10240"; OUR_RUNS=50; CUBLAS_RUNS=20; WARMUPS=5 ;;
  *) echo "--preset must be quick or paper" >&2; exit 2 ;;
esac

run() { printf '[l2d] +'; printf ' %q' "$@"; printf '\n'; (( DRY_RUN )) || "$@"; }

if [[ "${OUTPUT_ARG}" == /* ]]; then OUT_DIR="$(realpath -m -- "${OUTPUT_ARG}")"; else OUT_DIR="$(realpath -m -- "${APP_DIR}/${OUTPUT_ARG}")"; fi
BIN_DIR="${PKG_DIR}/bin"
OURS_BIN="${BIN_DIR}/gemv_sidegpu_l32_w16"
CUBLAS_BIN="${BIN_DIR}/gemv_cublas_benchmark"

run make -s -C "${PKG_DIR}/csrc" all
(( BUILD_ONLY )) && exit 0

# GPU selection and an exclusive lock per GPU (flock), as the reference runner holds one.
if (( DRY_RUN )); then
  GPU_INDEX="${DEVICE}"; [[ "${GPU_INDEX}" != auto ]] || GPU_INDEX="<auto-selected-physical-index>"
  GPU_NAME="dry-run"
else
  command -v nvidia-smi >/dev/null || { echo "nvidia-smi not found" >&2; exit 1; }
  mapfile -t GPUS < <(nvidia-smi --query-gpu=index,uuid,name --format=csv,noheader)
  GPU_INDEX="" GPU_NAME=""
  deadline=$(( $(date +%s) + WAIT_TIMEOUT ))
  while [[ -z "${GPU_INDEX}" ]]; do
    for line in "${GPUS[@]}"; do
      idx="${line%%,*}"; rest="${line#*, }"; uuid="${rest%%,*}"; name="${rest#*, }"
      [[ "${DEVICE}" == auto || "${DEVICE}" == "${idx}" || "${DEVICE}" == "${uuid}" ]] || continue
      exec {LOCK_FD}>"/tmp/l2d-gpu-${uuid//[^A-Za-z0-9_.-]/_}.lock"
      if flock -n "${LOCK_FD}"; then GPU_INDEX="${idx}"; GPU_NAME="${name}"; break; fi
      exec {LOCK_FD}>&-
    done
    [[ -n "${GPU_INDEX}" ]] && break
    (( $(date +%s) < deadline )) || { echo "timed out waiting for GPU '${DEVICE}'" >&2; exit 1; }
    sleep "${POLL_INTERVAL}"
  done
fi
case "${GPU_NAME}" in *B200*) GPU_CSV_NAME="B200" ;; *) GPU_CSV_NAME="CUSTOM" ;; esac
run mkdir -p "${OUT_DIR}"
export SIDEDGPU_CONFIG_DIR="${OUT_DIR}/config"
run mkdir -p "${SIDEDGPU_CONFIG_DIR}"
gpu() { run env "CUDA_VISIBLE_DEVICES=${GPU_INDEX}" "SIDEDGPU_CONFIG_DIR=${SIDEDGPU_CONFIG_DIR}" "$@"; }

if (( DRY_RUN )); then
  for m in ${M_VALUES}; do
    gpu "${OURS_BIN}" "${m}" "${OUR_RUNS}" 4242 1 "${K}" "${DTYPE}"
    gpu "${CUBLAS_BIN}" "${m}" "${K}" "${CUBLAS_RUNS}" "${WARMUPS}" 1 "${DTYPE}"
  done
  run python3 "${APP_DIR}/plot_gemv.py" --data-dir "${OUT_DIR}" --output-dir "${OUT_DIR}"
  exit 0
fi

TOL=0.001; [[ "${DTYPE}" == fp32 ]] || TOL=0.02
CSV="${OUT_DIR}/final_gemv_${GPU_CSV_NAME}.csv"
echo "M,K,lanes_per_row,warps_per_block,baseline_ms,aware_ms,swapped_ms,cublas_ms,max_abs_error,aware_speedup,swapped_speedup,aware_vs_cublas,pass,dtype,aware_gbs" > "${CSV}"
python3 - "${OUT_DIR}/metadata.json" "${GPU_INDEX}" "${GPU_NAME}" "${PRESET}" "${DTYPE}" "${K}" <<'PY'
import json, sys, datetime
out, idx, name, preset, dtype, k = sys.argv[1:]
json.dump({"timestamp_utc": datetime.datetime.now(datetime.timezone.utc).isoformat(), "application": "gemv",
           "preset": preset, "dtype": dtype, "K": int(k), "gpu": {"physical_index": idx, "name": name},
           "arch": "sm_100a"}, open(out, "w"), indent=2)
PY
parse_value() { awk -v p="$1" '$1 == p {print $2; exit}' "$2"; }
FAILURES=0
for m in ${M_VALUES}; do
  ours_log="${OUT_DIR}/.gemv_${m}_ours.log"; cublas_log="${OUT_DIR}/.gemv_${m}_cublas.log"
  echo "===== M=${m} K=${K} ${DTYPE} ====="
  set +e
  gpu "${OURS_BIN}" "${m}" "${OUR_RUNS}" 4242 1 "${K}" "${DTYPE}" 2>&1 | tee "${ours_log}"; os="${PIPESTATUS[0]}"
  gpu "${CUBLAS_BIN}" "${m}" "${K}" "${CUBLAS_RUNS}" "${WARMUPS}" 1 "${DTYPE}" 2>&1 | tee "${cublas_log}"; cs="${PIPESTATUS[0]}"
  set -e
  b="$(parse_value baseline_ms "${ours_log}")"; a="$(parse_value aware_ms "${ours_log}")"
  s="$(parse_value swapped_ms "${ours_log}")"; c="$(parse_value cublas_ms "${cublas_log}")"
  e="$(awk '/correctness max_abs_error/{max=0; for(i=1;i<=NF;i++) if($i~/=/){split($i,q,"="); if((q[2]+0)>max)max=q[2]+0} print max; exit}' "${ours_log}")"
  eb=4; [[ "${DTYPE}" == fp32 ]] || eb=2
  row="$(awk -v b="$b" -v a="$a" -v s="$s" -v c="$c" -v e="$e" -v os="$os" -v cs="$cs" -v tol="$TOL" \
        -v m="$m" -v k="$K" -v eb="$eb" -v dt="$DTYPE" 'BEGIN {
      ok = (os==0 && cs==0 && b>0 && a>0 && s>0 && c>0 && e!="" && e+0<=tol)
      gbs = (a>0) ? (m*k*eb + k*eb + m*eb) / (a*1e-3) / 1e9 : 0
      printf "%d,%d,32,16,%s,%s,%s,%s,%s,%.9f,%.9f,%.9f,%s,%s,%.3f", m, k, b, a, s, c, e,
             (a>0?b/a:0), (s>0?b/s:0), (a>0?c/a:0), ok ? "PASS" : "FAIL", dt, gbs }')"
  echo "${row}" >> "${CSV}"
  [[ "${row}" == *",PASS,"* ]] || FAILURES=$((FAILURES + 1))
  rm -f "${ours_log}" "${cublas_log}"
done
if (( FAILURES > 0 )); then echo "CSV: ${CSV}"; echo "${FAILURES} benchmark case(s) failed" >&2; exit 1; fi
run python3 "${APP_DIR}/plot_gemv.py" --data-dir "${OUT_DIR}" --output-dir "${OUT_DIR}"
echo "CSV: ${CSV}"
