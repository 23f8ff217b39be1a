"""Markdown report over gemm_bench's bench.csv and bench.py's JSON lines.

The reference turns results/bench.csv into charts plus a summary table (analysis/plot.py:1-48,
report.md). This module reads the same CSV schema (device,sm,M,N,K,kernel,ms,tflops,
pct_of_cublas,max_abs_err, src/main.cu:103; gemm_bench appends pct_of_peak,dtype, which older
files lack) and adds what the B200 build measures beside it: each row against the library
kernel of the same precision, and the GPU-count dimension from bench.py's JSON lines (one per
run, N = 1..8). No plotting library is needed: the output is Markdown tables.

    python report.py results/bench.csv [--bench-json runs.jsonl] [--out report.md]
"""
from __future__ import annotations

import argparse
import collections
import csv
import json

# same-precision library row for each of this repo's rows (and the reference's)
LIBRARY_OF = {
    "tc_f16": "cublas_tc", "ref_mma_warptile": "cublas_tc", "ref_wmma": "cublas_tc",
    "tc_fp8": "cublaslt_fp8", "ref_mma_fp8": "cublaslt_fp8", "tc_fp8_amax": "cublaslt_fp8_amax",
    "tc_mxfp4_b32": "cublaslt_mxfp4",
}
ORDER = ["tc_f16", "tc_fp8", "tc_fp8_amax", "tc_fp4", "tc_fp4_amax", "tc_mxfp4", "tc_mxfp4_b32",
         "ref_wmma", "ref_mma_warptile", "ref_mma_fp8",
         "cublas", "cublas_tc", "cublaslt_fp8", "cublaslt_fp8_amax", "cublaslt_mxfp4"]


def load_csv(path: str) -> list[dict]:
    with open(path) as f:
        return list(csv.DictReader(f))


def load_json_lines(path: str) -> list[dict]:
    out = []
    with open(path) as f:
        for line in f:
            line = line.strip()
            if line.startswith("{"):
                out.append(json.loads(line))
    return out


def _rank(kernel: str) -> int:
    return ORDER.index(kernel) if kernel in ORDER else len(ORDER)


def size_tables(rows: list[dict]) -> list[str]:
    """One table per (device, problem size): throughput, % of the same-precision library row,
    % of the dtype's nominal dense peak, and the error the driver measured."""
    by = collections.defaultdict(dict)
    for r in rows:
        key = (r["device"], r["sm"], int(r["M"]), int(r["N"]), int(r["K"]))
        by[key][r["kernel"]] = r  # a later run of the same row replaces an earlier one
    lines = []
    for (dev, sm, M, N, K) in sorted(by, key=lambda k: (k[0], k[1], k[2] * k[3] * k[4], k[2])):
        kerns = by[(dev, sm, M, N, K)]
        lines += [f"### {dev} (sm_{sm}), M = {M}, N = {N}, K = {K}", "",
                  "| kernel | dtype | TFLOP/s | % of same-precision library | % of dense peak | max abs err |",
                  "|---|---|---|---|---|---|"]
        for k in sorted(kerns, key=lambda k: (_rank(k), k)):
            r = kerns[k]
            tf = float(r["tflops"])
            lib = LIBRARY_OF.get(k)
            pct = f"{100.0 * tf / float(kerns[lib]['tflops']):.1f}% of {lib}" if lib in kerns else "-"
            peak = f"{float(r['pct_of_peak']):.1f}%" if r.get("pct_of_peak") else "-"
            lines.append(f"| {k} | {r.get('dtype') or '-'} | {tf:.1f} | {pct} | {peak} | "
                         f"{float(r['max_abs_err']):.3g} |")
        lines.append("")
    return lines


def scaling_table(runs: list[dict]) -> list[str]:
    """bench.py lines grouped by workload: whole-box TFLOP/s per GPU count, the ratio to the
    one-GPU line of the same workload, and the gather columns when present."""
    groups = collections.defaultdict(list)
    for d in runs:
        if "unavailable" in d or d.get("impl", "ours") != "ours":
            continue
        groups[d.get("config", {}).get("workload", "?")].append(d)
    lines = []
    for wl in sorted(groups):
        ds = sorted(groups[wl], key=lambda d: d["n_gpus"])
        base = next((d["value"] for d in ds if d["n_gpus"] == 1), None)
        lines += [f"### {wl}", "",
                  "| GPUs | TFLOP/s (all GPUs) | x one GPU | ms per step | e2e TFLOP/s | NCCL gather ms | fused GEMM+gather ms |",
                  "|---|---|---|---|---|---|---|"]
        for d in ds:
            g = d.get("gather") or {}
            fused = g.get("fused") or {}
            ratio = f"{d['value'] / base:.2f}" if base else "-"
            e2e = (d.get("e2e") or {}).get("value", "-")
            lines.append(f"| {d['n_gpus']} | {d['value']:.1f} | {ratio} | {d['ms_per_step']} | {e2e} | "
                         f"{g.get('ms', '-')} | {fused.get('ms_per_step', '-')} |")
        lines.append("")
    return lines


def render(csv_rows: list[dict], runs: list[dict]) -> str:
    out = ["# GEMM report", ""]
    if csv_rows:
        out += ["## gemm_bench rows", ""] + size_tables(csv_rows)
    if runs:
        out += ["## bench.py runs by GPU count", ""] + scaling_table(runs)
    return "\n".join(out) + "\n"


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("csv", nargs="?", help="gemm_bench output (bench.csv schema)")
    ap.add_argument("--bench-json", action="append", default=[], help="file of bench.py JSON lines (repeatable)")
    ap.add_argument("--out", help="write here instead of stdout")
    a = ap.parse_args(argv)
    rows = load_csv(a.csv) if a.csv else []
    runs = [d for p in a.bench_json for d in load_json_lines(p)]
    text = render(rows, runs)
    if a.out:
        with open(a.out, "w") as f:
            f.write(text)
    else:
        print(text, end="")


if __name__ == "__main__":
    main()
