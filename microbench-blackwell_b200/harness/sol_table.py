#!/usr/bin/env python3
"""Speed-of-light table (and, where matplotlib exists, plots) of a mainloop sweep.

Extends what the reference's cutlass_gemm_mainloop/plot_results.py computes
(:22-27 per-SM peak = FLOP/clk/SM x 1300 MHz for BF16 and FP8_E4M3 only; :42-43
pct_sol) to every row of results.csv, NVFP4 and CTA-pair tiles included, and
adds a second SOL against *measured* numbers:

  pct_sol_1300      the reference's formula, with NVFP4 at 32768 FLOP/clk/SM and a
                    CTA pair (TILE_M 256) counted as two SMs;
  pct_sol_measured  TFLOPS over (the own tcgen05 probe's FLOP/clk/SM for the dtype,
                    x SMs, x the SM clock the point itself ran at -- the sm_mhz
                    column the in-process sweep records); a point at the tensor
                    pipe's rate reads 100 whatever the clock;
  vs_published      TFLOPS over the reference's own published result for the same
                    (TILE_M, TILE_N, TILE_K, STAGES, dtype), when its results.csv is
                    given.

Usage: sol_table.py results.csv [--peaks peaks.json] [--reference-results ref.csv]
                    [--markdown out.md] [--plots]
peaks.json: {"BF16": f, "FP8_E4M3": f, "NVFP4": f} measured FLOP/clk/SM; without it
the probe runs here when a GPU is present, else the nominal rates are used and the
table says so.
"""
from __future__ import annotations

import argparse
import json
import sys
from io import StringIO
from pathlib import Path

NOMINAL_FLOP_PER_CLK_SM = {"BF16": 8192.0, "FP8_E4M3": 16384.0, "NVFP4": 32768.0}
REFERENCE_CLOCK_MHZ = 1300.0                        # plot_results.py:22


def read_results(path) -> "pandas.DataFrame":
    import pandas as pd
    lines = [l for l in Path(path).read_text().splitlines() if l.strip() and not l.startswith("#")]
    return pd.read_csv(StringIO("\n".join(lines)))


def with_sol(df, flop_per_clk_sm: dict, published=None):
    """Add the SOL columns to a results data frame (one row per measured point)."""
    df = df.copy()
    df["tile_label"] = [f"{int(m)}x{int(n)}x{int(k)}" for m, n, k in zip(df.TILE_M, df.TILE_N, df.TILE_K)]
    df["sms"] = [2 if int(m) > 128 else 1 for m in df.TILE_M]
    nominal = df["dtype"].map(NOMINAL_FLOP_PER_CLK_SM)
    df["peak_1300"] = nominal * df["sms"] * REFERENCE_CLOCK_MHZ * 1e6 / 1e12
    df["pct_sol_1300"] = 100.0 * df["TFLOPS"] / df["peak_1300"]
    if "sm_mhz" in df.columns:
        rate = df["dtype"].map(flop_per_clk_sm)
        df["peak_measured"] = rate * df["sms"] * df["sm_mhz"] * 1e6 / 1e12
        df["pct_sol_measured"] = 100.0 * df["TFLOPS"] / df["peak_measured"]
    if published is not None:
        key = ["TILE_M", "TILE_N", "TILE_K", "STAGES", "dtype"]
        ref = published[key + ["TFLOPS"]].rename(columns={"TFLOPS": "published_TFLOPS"})
        df = df.merge(ref, on=key, how="left")
        df["vs_published"] = df["TFLOPS"] / df["published_TFLOPS"]
    return df


def best_per_tile(df):
    """The fastest stage count of every tile, as the reference's plots pick it."""
    idx = df.groupby(["dtype", "tile_label"])["TFLOPS"].idxmax()
    return df.loc[idx].sort_values(["dtype", "TILE_M", "TILE_N", "TILE_K"])


def measure_rates():
    """Per-SM FLOP/clk of one CTA (1SM, M128 N256) from the library's tcgen05 probe."""
    import importlib.util
    pkg_dir = Path(__file__).resolve().parent.parent
    spec = importlib.util.spec_from_file_location("microbench_blackwell_b200", pkg_dir / "__init__.py",
                                                  submodule_search_locations=[str(pkg_dir)])
    pkg = importlib.util.module_from_spec(spec)
    sys.modules[spec.name] = pkg
    spec.loader.exec_module(pkg)
    return {name: pkg.umma_peak(dt, cta_group=1, num_ctas=1, depth=256, iters=400)["flop_per_clk_per_sm"]
            for dt, name in ((pkg.BF16, "BF16"), (pkg.FP8_E4M3, "FP8_E4M3"), (pkg.NVFP4, "NVFP4"))}


def markdown(df, rates_note: str) -> str:
    cols = ["dtype", "tile_label", "STAGES", "TFLOPS", "pct_sol_1300"]
    cols += [c for c in ("sm_mhz", "pct_sol_measured", "published_TFLOPS", "vs_published") if c in df.columns]
    out = [f"FLOP/clk/SM used for pct_sol_measured: {rates_note}", "",
           "| " + " | ".join(cols) + " |", "|" + "---|" * len(cols)]
    for _, r in df.iterrows():
        cells = []
        for c in cols:
            v = r[c]
            cells.append(f"{v:.3g}" if isinstance(v, float) else str(v))
        out.append("| " + " | ".join(cells) + " |")
    return "\n".join(out) + "\n"


def plots(df, outdir: Path):
    try:
        import matplotlib.pyplot as plt
    except ImportError:
        print("matplotlib is not installed: table only", file=sys.stderr)
        return
    col = "pct_sol_measured" if "pct_sol_measured" in df.columns else "pct_sol_1300"
    dts = sorted(df["dtype"].unique())
    fig, axes = plt.subplots(1, len(dts), figsize=(8 * len(dts), 6))
    for ax, dt in zip(axes if len(dts) > 1 else [axes], dts):
        sub = df[(df["dtype"] == dt) & (df["STAGES"] != 0)]
        for tile in sorted(sub["tile_label"].unique()):
            t = sub[sub["tile_label"] == tile].sort_values("STAGES")
            ax.plot(t["STAGES"], t[col], "o-", label=tile, markersize=4)
        ax.axhline(100, color="red", linestyle="--")
        ax.set_title(f"{dt}: {col} vs stages")
        ax.set_xlabel("stages")
        ax.legend(fontsize=6, ncol=2)
    fig.tight_layout()
    fig.savefig(outdir / "sol_vs_stages.png", dpi=120)


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("results")
    ap.add_argument("--peaks", help="JSON of measured FLOP/clk/SM per dtype")
    ap.add_argument("--reference-results", help="the reference's published results.csv")
    ap.add_argument("--markdown", help="write the best-per-tile table here")
    ap.add_argument("--plots", action="store_true")
    args = ap.parse_args()
    if args.peaks:
        rates, note = json.loads(Path(args.peaks).read_text()), f"measured ({args.peaks})"
    else:
        try:
            rates, note = measure_rates(), "measured now by gemm_sm100a_umma_peak (1 CTA, M128 N256)"
        except Exception as e:  # no GPU here
            rates, note = dict(NOMINAL_FLOP_PER_CLK_SM), f"nominal (probe unavailable: {type(e).__name__})"
    df = read_results(args.results)
    pub = read_results(args.reference_results) if args.reference_results else None
    full = with_sol(df, rates, pub)
    best = best_per_tile(full)
    text = markdown(best, note)
    if args.markdown:
        Path(args.markdown).write_text(text)
    print(text)
    if args.plots:
        plots(full, Path(args.results).resolve().parent)


if __name__ == "__main__":
    main()
