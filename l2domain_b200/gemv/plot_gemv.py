#!/usr/bin/env python3
"""Validate (and, when matplotlib is installed, plot) final_gemv_*.csv files.

Validation follows the reference's plot gate (applications/gemv/plot_gemv.py:36-54): no empty
file, every row pass=PASS, one lanes/warps configuration.  The reference also demands K=1024; this
build accepts any K but requires one K (and one dtype) per file.  Without matplotlib the CSVs are
validated and a text summary is printed instead of figure_11.png/.pdf.
"""
import argparse
import csv
import sys
from pathlib import Path

INT_COLS = {"M", "K", "lanes_per_row", "warps_per_block"}
TEXT_COLS = {"pass", "dtype"}


def load_csv(path: Path):
    with path.open() as f:
        return [{k: (int(v) if k in INT_COLS else v if k in TEXT_COLS else float(v)) for k, v in row.items()}
                for row in csv.DictReader(f)]


def validate_rows(path: Path, rows, expected_config=None):
    if not rows:
        raise ValueError(f"{path}: CSV contains no data rows")
    ks = {r["K"] for r in rows}
    if len(ks) != 1:
        raise ValueError(f"{path}: mixed K values {sorted(ks)}")
    for n, row in enumerate(rows, start=2):
        if row["pass"] != "PASS":
            raise ValueError(f"{path}:{n}: refusing to plot pass={row['pass']}")
        cfg = (row["lanes_per_row"], row["warps_per_block"])
        if expected_config is None:
            expected_config = cfg
        elif cfg != expected_config:
            raise ValueError(f"{path}:{n}: mixed GEMV configurations {expected_config} vs {cfg}")
    return expected_config


def main(argv=None):
    ap = argparse.ArgumentParser(description="Validate/plot final GEMV CSVs.")
    ap.add_argument("--data-dir", default="out")
    ap.add_argument("--output-dir", default="out")
    args = ap.parse_args(argv)
    files = sorted(Path(args.data_dir).glob("final_gemv_*.csv"))
    if not files:
        ap.error(f"no GEMV CSVs found in {args.data_dir}")
    loaded, cfg = [], None
    for f in files:
        rows = load_csv(f)
        cfg = validate_rows(f, rows, cfg)
        loaded.append((f.stem.removeprefix("final_gemv_"), rows))
    try:
        import matplotlib
        matplotlib.use("Agg")
        import matplotlib.pyplot as plt
    except ImportError:
        for title, rows in loaded:
            print(f"{title}: " + ", ".join(f"M={r['M']} aware={r['aware_ms'] * 1e3:.2f}us "
                                          f"baseline={r['baseline_ms'] * 1e3:.2f}us" for r in rows))
        print("matplotlib unavailable: CSVs validated, no figure written")
        return 0
    out = Path(args.output_dir)
    out.mkdir(parents=True, exist_ok=True)
    fig, axes = plt.subplots(1, len(loaded), figsize=(5.6 * len(loaded), 6), squeeze=False)
    for ax, (title, rows) in zip(axes[0], loaded):
        for key, marker in (("aware_ms", "o"), ("baseline_ms", "s"), ("swapped_ms", "^"), ("cublas_ms", "D")):
            ax.plot([r["M"] for r in rows], [r[key] * 1e3 for r in rows], marker=marker, label=key[:-3])
        ax.set_title(title)
        ax.set_xlabel(f"M (rows), K={rows[0]['K']}")
        ax.set_ylabel("Time (us)")
        ax.grid(True, alpha=0.3)
    axes[0][0].legend()
    fig.savefig(out / "figure_11.png", dpi=160, bbox_inches="tight")
    fig.savefig(out / "figure_11.pdf", bbox_inches="tight")
    print(f"Saved {out / 'figure_11.png'} and {out / 'figure_11.pdf'}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
